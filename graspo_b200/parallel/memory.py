"""Memory budgeting for pipelined micro-batches.

``estimate_per_microbatch_activation_bytes`` counts what one micro-batch keeps
alive on a stage under whole-layer recomputation: the input of every local
layer plus one layer's worth of transient intermediates (the layer being
recomputed in backward).  ``compute_max_inflight`` turns free device memory
into a bound on concurrently live micro-batches with a safety factor
(reference: backends/graspoflow/memory.py:11-98).
"""

from __future__ import annotations

import torch


def estimate_per_microbatch_activation_bytes(
    *,
    batch_size: int,
    seq_len: int,
    hidden_size: int,
    intermediate_size: int,
    num_local_layers: int,
    tp_size: int = 1,
    dtype_bytes: int = 2,
    recompute: bool = True,
) -> int:
    tokens = int(batch_size) * int(seq_len)
    layer_inputs = tokens * hidden_size * dtype_bytes * num_local_layers
    # one layer's saved set: ~6 hidden-sized tensors + gate/up pre-activations + SwiGLU output
    per_layer = tokens * dtype_bytes * (6 * hidden_size + 3 * intermediate_size // tp_size)
    if recompute:
        return layer_inputs + per_layer
    return layer_inputs + per_layer * num_local_layers


def get_gpu_free_memory_bytes(device: int | None = None) -> int:
    if not torch.cuda.is_available():
        return 0
    free, _ = torch.cuda.mem_get_info(device if device is not None else torch.cuda.current_device())
    return int(free)


def compute_max_inflight(
    *,
    per_microbatch_bytes: int,
    free_bytes: int | None = None,
    reserve_bytes: int = 2 << 30,
    safety: float = 0.8,
    hard_cap: int = 64,
) -> int:
    free = get_gpu_free_memory_bytes() if free_bytes is None else int(free_bytes)
    budget = int(max(0, free - reserve_bytes) * safety)
    if per_microbatch_bytes <= 0:
        return hard_cap
    return max(1, min(hard_cap, budget // int(per_microbatch_bytes)))
