"""Safetensors checkpoint access that reads only the bytes a rank needs.

The reference loads each shard file whole onto the CPU and slices it per rank
(reference: tensor_utils.py:28-57).  Here tensors are opened lazily through
``safe_open`` and sliced before materialisation, so a TP rank reading its
1/tp slice of a 12288-wide matrix touches only that slice, and nothing is
cached beyond the file handles.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors import safe_open


class SafetensorIndex:
    def __init__(self, model_path: str | Path) -> None:
        self.model_path = Path(model_path)
        self.weight_map: dict[str, str] = {}
        index = self.model_path / "model.safetensors.index.json"
        if index.exists():
            self.weight_map = dict(json.loads(index.read_text(encoding="utf-8"))["weight_map"])
        else:
            files = sorted(self.model_path.glob("*.safetensors"))
            if not files:
                raise FileNotFoundError(f"No safetensors files found in {self.model_path}")
            for file in files:
                with safe_open(str(file), framework="pt") as handle:
                    for key in handle.keys():
                        self.weight_map[key] = file.name
        self._handles: dict[str, object] = {}

    def _handle(self, filename: str):
        handle = self._handles.get(filename)
        if handle is None:
            handle = safe_open(str(self.model_path / filename), framework="pt")
            self._handles[filename] = handle
        return handle

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def get(self, name: str) -> torch.Tensor:
        value = self.get_optional(name)
        if value is None:
            raise KeyError(f"Tensor not found in HF checkpoint: {name}")
        return value

    def get_optional(self, name: str) -> torch.Tensor | None:
        filename = self.weight_map.get(name)
        if filename is None:
            return None
        return self._handle(filename).get_tensor(name)

    def get_rows(self, name: str, start: int, stop: int) -> torch.Tensor:
        """Rows [start, stop) of a 1-D or 2-D tensor, reading only that slice."""
        filename = self.weight_map[name]
        return self._handle(filename).get_slice(name)[start:stop]

    def get_cols(self, name: str, start: int, stop: int) -> torch.Tensor:
        filename = self.weight_map[name]
        return self._handle(filename).get_slice(name)[:, start:stop]

    def close(self) -> None:
        self._handles.clear()


def shard_bounds(size: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous equal split; ``size`` must divide by ``world``."""
    if size % world:
        raise ValueError(f"Cannot shard size {size} by TP={world}")
    chunk = size // world
    return rank * chunk, (rank + 1) * chunk
