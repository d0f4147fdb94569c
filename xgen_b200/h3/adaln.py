"""AdaLN sources of the H3 block: schedule tables, the rank-owner projection,
modality row indices, and the local sequence span.

- `AdalnScheduleCache` mirrors x_base/x_base/adaln_cache/cache.py:47-296:
  precomputed modulation tables keyed by the float32 bits of the timestep
  schedule, read from a safetensors file (bf16, or int8 + fp32 scale), with
  the constant condition rows (0.999, 1.0) pre-merged per conditioning type.
  `lookup_block(i)` returns the 6 [M*3, H] modulation tensors of block i
  (shift, scale, gate, shift_ff, scale_ff, gate_ff), views of one
  [M*3, 6H] table that `lookup_block_table(i)` returns whole for
  `H3DiTBlockB200.forward`; `lookup_final()` returns the final layer's
  (shift, scale).
- `H3OwnedAdaLN` mirrors x_base/x_base/operator/h3_adaln_owner.py:9-41: one
  SP rank per block computes linear(silu(temb)) and broadcasts it.
- `adaln_indices` is minimax_h3.py:410-415: row = t_idx * 3 + modality tag,
  plus the pad mask of negative tags.
- `LocalSpan` (defined in h3/local_io.py, re-exported here) is the rank's
  block of the packed sequence, x_diffusers/.../h3_local_io.py:14-38.

safetensors is not a dependency: `SafetensorsFile` / `write_safetensors`
implement its published layout (little-endian u64 header length, a JSON
header of {name: {dtype, shape, data_offsets}} plus "__metadata__", then the
raw tensor bytes).
"""
from __future__ import annotations

import json
import logging
import os
import struct
import numpy as np
import torch
import torch.distributed as dist
from torch import nn

from .local_io import LocalSpan  # noqa: F401  (re-exported)

logger = logging.getLogger(__name__)

MODALITY_NUM = 3  # video, audio, text rows per timestep (MINIMAX_H3_MODALITY_NUM)

_DTYPES = {
    "BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "F64": torch.float64,
    "I8": torch.int8, "U8": torch.uint8, "I16": torch.int16, "I32": torch.int32,
    "I64": torch.int64, "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


class SafetensorsFile:
    """Read-only view of a safetensors file (the data section is memory-mapped)."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
        self._meta = header.pop("__metadata__", None) or {}
        self._entries = header
        self._data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)

    def keys(self):
        return list(self._entries)

    def metadata(self) -> dict:
        return dict(self._meta)

    def get_tensor(self, name: str) -> torch.Tensor:
        e = self._entries[name]
        begin, end = e["data_offsets"]
        dtype = _DTYPES[e["dtype"]]
        raw = torch.from_numpy(np.array(self._data[begin:end]))
        return raw.view(dtype).reshape(e["shape"])


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    header, offset, blobs = {}, 0, []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        blob = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [offset, offset + len(blob)]}
        offset += len(blob)
        blobs.append(blob)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for blob in blobs:
            f.write(blob)


class AdalnScheduleCache:
    """AdaLN modulation tables keyed by timestep schedule (file cache mode)."""

    # const_timesteps = [0.999, 1.0]: index 0 = video, 1 = audio conditioning.
    _CONST_INDEX_MAP = {"none": [], "video": [0], "audio": [1], "both": [0, 1]}

    def __init__(self, num_blocks: int | None = None, cache_file: str | None = None,
                 conditioning_type: str = "none", device="cuda"):
        self.num_blocks = num_blocks
        self._tables = {}
        self._current_key = None
        self._current_table = None
        self._file_cache_loaded = False
        self._const_table = None
        self._const_timesteps = None
        self._conditioning_type = conditioning_type
        self._source_file = os.path.realpath(cache_file) if cache_file else None
        self._device = torch.device(device)
        if cache_file:
            self._load_file_cache(cache_file)

    # -- file cache loading (cache.py:84-186)
    def _load_file_cache(self, path: str):
        f = SafetensorsFile(path)
        metadata = f.metadata()
        # Older tables record only num_steps (sigma points, terminal 0 included).
        num_eval_steps = int(metadata["num_eval_steps"]) if "num_eval_steps" in metadata \
            else int(metadata["num_steps"]) - 1
        num_blocks = int(metadata.get("num_blocks", self.num_blocks or 0))
        if num_blocks <= 0:
            raise ValueError("AdaLN table does not record num_blocks and none was given")
        self.num_blocks = num_blocks
        quantization = metadata.get("quantization", "none")
        conditioned = metadata.get("conditioning_tables")
        if conditioned and self._conditioning_type not in conditioned.split(","):
            raise ValueError(f"AdaLN table does not contain conditioning={self._conditioning_type}")
        prefix = f"{self._conditioning_type}_" if conditioned else ""

        step_entries = []
        for step_idx in range(num_eval_steps):
            ts = f.get_tensor(f"{prefix}step{step_idx}_timesteps").to(self._device)
            blocks = [self._split_block(self._read_tensor(f, f"{prefix}step{step_idx}_block{b}", quantization))
                      for b in range(num_blocks)]
            final = self._read_tensor(f, f"{prefix}step{step_idx}_final", quantization).chunk(2, dim=-1)
            step_entries.append((ts, {"blocks": blocks, "final": final}))

        if "const_timesteps" in f.keys():
            self._const_timesteps = f.get_tensor("const_timesteps").to(self._device)
            self._const_table = {
                "blocks": [self._split_block(self._read_tensor(f, f"const_block{b}", quantization))
                           for b in range(num_blocks)],
                "final": self._read_tensor(f, "const_final", quantization).chunk(2, dim=-1),
            }
        elif not conditioned:
            logger.warning("No constant timesteps in cache file. "
                           "Condition row (0.999, 1.0) cache miss will error.")

        const_indices = [] if conditioned else self._CONST_INDEX_MAP.get(self._conditioning_type, [])
        if const_indices:
            if self._const_table is None:
                raise RuntimeError(f"conditioning_type={self._conditioning_type} requires constant "
                                   "entries but the cache file has none")
            const_sel = torch.tensor(const_indices, dtype=torch.long, device=self._device)
            const_ts = self._const_timesteps[const_indices]
            for step_ts, table in step_entries:
                key = self._schedule_key(torch.cat([step_ts, const_ts]))
                self._tables[key] = self._merge_table(table, const_sel)
        else:
            for step_ts, table in step_entries:
                self._tables[self._schedule_key(step_ts)] = table
        self._file_cache_loaded = True
        logger.info("AdaLN cache loaded: %d steps, %d blocks, %d tables, conditioning=%s, quant=%s",
                    num_eval_steps, num_blocks, len(self._tables), self._conditioning_type,
                    quantization)

    @staticmethod
    def _split_block(raw: torch.Tensor):
        # raw [M, 3*6*H] -> [M*3, 6H] -> 6 views [M*3, H] (cache.py:112-116)
        width = raw.shape[-1] // (6 * MODALITY_NUM)
        return raw.view(-1, 6 * width).chunk(6, dim=-1)

    def _read_tensor(self, f: SafetensorsFile, key: str, quantization: str) -> torch.Tensor:
        """bf16 table, or int8 codes times an fp32 scale rounded to bf16 (cache.py:188-200)."""
        if quantization == "int8":
            codes = f.get_tensor(f"{key}_int8").to(self._device)
            scale = f.get_tensor(f"{key}_scale").to(self._device)
            return (codes.to(torch.float32) * scale).to(torch.bfloat16)
        return f.get_tensor(key).to(self._device)

    def _merge_table(self, step_table: dict, const_sel: torch.Tensor) -> dict:
        """Step rows, then the selected constant rows (cache.py:204-259)."""
        row_sel = (const_sel.unsqueeze(1) * MODALITY_NUM
                   + torch.arange(MODALITY_NUM, device=const_sel.device)).reshape(-1)
        blocks = []
        for step_mod, const_mod in zip(step_table["blocks"], self._const_table["blocks"]):
            # one contiguous [rows, 6H] table whose 6 chunks are the merged tensors
            merged = torch.cat([torch.cat(step_mod, dim=-1),
                                torch.cat([c.index_select(0, row_sel) for c in const_mod], dim=-1)])
            blocks.append(merged.chunk(6, dim=-1))
        shift = torch.cat([step_table["final"][0], self._const_table["final"][0].index_select(0, const_sel)])
        scale = torch.cat([step_table["final"][1], self._const_table["final"][1].index_select(0, const_sel)])
        return {"blocks": blocks, "final": (shift, scale)}

    @staticmethod
    def _schedule_key(timesteps: torch.Tensor) -> bytes:
        """Float32 bit pattern of the timesteps (cache.py:263-267)."""
        return timesteps.to(torch.float32).cpu().numpy().tobytes()

    # -- install / lookup (cache.py:271-296)
    def maybe_install(self, timesteps: torch.Tensor):
        key = self._schedule_key(timesteps)
        if key == self._current_key:
            return
        self._current_table = self._tables[key]
        self._current_key = key

    @property
    def has_current(self) -> bool:
        return self._current_table is not None

    def lookup_block(self, block_idx: int):
        """6 tensors [M*3, H]: shift, scale, gate, shift_ff, scale_ff, gate_ff."""
        return self._current_table["blocks"][block_idx]

    def lookup_block_table(self, block_idx: int) -> torch.Tensor:
        """The [M*3, 6H] table the 6 lookup_block tensors are views of."""
        first = self._current_table["blocks"][block_idx][0]
        return first.as_strided((first.shape[0], first.stride(0)), (first.stride(0), 1))

    def lookup_final(self):
        """(shift, scale), each [M, H]."""
        return self._current_table["final"]


def adaln_indices(timestep_indices: torch.Tensor, token_tags: torch.Tensor):
    """Table rows t_idx * 3 + tag and the attention mask of padded tokens
    (negative tags), as minimax_h3.py:410-415."""
    indices = timestep_indices * MODALITY_NUM + token_tags.clamp(min=0)
    is_pad = token_tags < 0
    mask = (is_pad[None, :] == is_pad[:, None]) if bool(is_pad.any()) else None
    return indices, mask


class H3OwnedAdaLN(nn.Module):
    """Block modulation computed on one SP rank (index % world) and broadcast
    to the others, with an optional exact-input cache on the owner."""

    def __init__(self, original, index: int, *, group=None, exact_cache: bool = False):
        super().__init__()
        self.group = group
        self.owner = index % dist.get_world_size(group)
        self.hidden_size = original.hidden_size
        self.out_features = original.linear.out_features
        self.output_dtype = original.linear.weight.dtype
        self.linear = original.linear if dist.get_rank(group) == self.owner else None
        self.exact_cache = exact_cache
        self.register_buffer("_last_input", None, persistent=False)
        self.register_buffer("_last_output", None, persistent=False)
        self.projection_calls = 0
        self.cache_hits = 0

    def forward(self, temb):
        if self.linear is not None:
            last = self._last_input
            if (self.exact_cache and last is not None and temb.dtype == last.dtype
                    and temb.device == last.device and torch.equal(temb, last)):
                output = self._last_output.clone()
                self.cache_hits += 1
            else:
                output = self.linear(nn.functional.silu(temb).to(self.linear.weight.dtype)).contiguous()
                self.projection_calls += 1
                if self.exact_cache:
                    self._last_input = temb.detach().clone()
                    self._last_output = output.detach().clone()
        else:
            output = torch.empty((*temb.shape[:-1], self.out_features), device=temb.device,
                                 dtype=self.output_dtype)
        src = dist.get_global_rank(self.group, self.owner) if self.group is not None else self.owner
        dist.broadcast(output, src=src, group=self.group)
        return output.reshape(-1, 6 * self.hidden_size).chunk(6, dim=-1)
