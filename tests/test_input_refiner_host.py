"""H3 input token refiner SP installer (xgen_b200/h3/input_refiner.py): the
argument and module checks of x_diffusers/x_diffusers/adaptor/
h3_input_refiner.py:67-86 and what installation changes, on CPU."""
from types import SimpleNamespace
from unittest.mock import patch

import pytest
import torch

from refiner_fakes import FakeRefiner
from xgen_b200.h3 import input_refiner as ir

DIST = "xgen_b200.h3.input_refiner.dist.get_world_size"


def _model(**kw):
    return SimpleNamespace(token_refiner=FakeRefiner(**kw))


def test_profile_attention_and_world_checks():
    with pytest.raises(ValueError, match="Unknown"):
        ir.install_input_refiner(_model(), "fp8")
    with patch(DIST, return_value=2):
        with pytest.raises(ValueError, match="only the B200 BF16 attention"):
            ir.install_input_refiner(_model(), "custom", attention="laser")
    with patch(DIST, return_value=3):
        with pytest.raises(ValueError, match="2/4/8 ranks"):
            ir.install_input_refiner(_model(), "cudnn-sp")
    with patch(DIST, return_value=4):  # 2 heads over 4 ranks
        with pytest.raises(ValueError, match="divisible attention heads"):
            ir.install_input_refiner(_model(), "cudnn-sp")


def test_dtype_and_double_install_checks():
    model = _model()
    model.token_refiner.float()
    with patch(DIST, return_value=2):
        with pytest.raises(ValueError, match="BF16 parameters"):
            ir.install_input_refiner(model, "cudnn-sp")
        model = _model()
        metrics = ir.install_input_refiner(model, "cudnn-sp")
        with pytest.raises(ValueError, match="already installed"):
            ir.install_input_refiner(model, "cudnn-sp")
    assert metrics["sp_size"] == 2 and metrics["ffn_precision"] == "bf16"
    assert model._h3_input_refiner_profile == "cudnn-sp"
    assert all(isinstance(b.attn.processor, ir.RefinerSPAttention) for b in model.token_refiner.refiner_blocks)


def test_forward_rejects_cpu_training_and_unbound_group():
    model = _model()
    with patch(DIST, return_value=2):
        ir.install_input_refiner(model, "cudnn-sp")
    x = torch.randn(1, 5, 256).bfloat16()
    with pytest.raises(ValueError, match="inference-only"):
        model.token_refiner(x)
    with torch.no_grad(), pytest.raises(ValueError, match="CUDA BF16"):
        model.token_refiner(x)
