"""Stage operators: the embedding, the local decoder layers and the LM head of
a model as ``ComputeOperator`` s that a ``PipelineGraph`` chains.

Each operator reads and writes named tensors of the ``Microbatch``:

* ``EmbedStageOp`` -- ``input_ids`` -> ``hidden`` (frozen table; an optional
  ``embed_hook`` in ``mb.meta`` places image features);
* ``DecoderStageOp`` -- ``hidden`` -> ``hidden`` through this rank's layers
  with the LoRA adapter as autograd leaves; its backward turns
  ``grad_hidden`` into the gradient of its input and adds the LoRA gradients
  into the adapter's flat gradient buffer (``finish``);
* ``HeadStageOp`` -- final norm + LM head -> ``logprobs`` of ``targets``;
  its backward takes ``grad_logprobs`` (d loss / d log-prob) and produces
  ``grad_hidden``.

Both model families are served: the dense Qwen3 model through its eager
layers, the Qwen3.5 hybrid through its stage forward.  The production
training and pipeline paths (``engine/pipeline.py``) do not go through these
operators; they exist for custom dataflow graphs (reference:
models/qwen3/ops.py:12-256, models/qwen35_36/ops.py:12-281,
transformer_op.py:27-107).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from graspo_b200.parallel.operator import ComputeOperator, Microbatch


def _is_hybrid(model) -> bool:
    return hasattr(model, "mrope_positions")


class EmbedStageOp(ComputeOperator):
    def __init__(self, model, *, name: str = "embed") -> None:
        super().__init__(name=name, tp_size=model.ps.tp_size)
        if model.embed is None:
            raise ValueError("EmbedStageOp needs a model stage that holds the embedding table")
        self.model = model

    def forward(self, mb: Microbatch) -> Microbatch:
        ids = mb.tensors["input_ids"]
        x = F.embedding(ids, self.model.embed)
        hook = mb.meta.get("embed_hook")
        if hook is not None:
            x = hook(ids, x.clone())
        mb.tensors["hidden"] = x
        return mb

    def backward(self, mb: Microbatch) -> Microbatch:
        mb.tensors.pop("grad_hidden", None)        # the table is frozen
        return mb


class DecoderStageOp(ComputeOperator):
    def __init__(self, model, *, training: bool = True, name: str = "decoder") -> None:
        super().__init__(name=name, tp_size=model.ps.tp_size)
        from graspo_b200.models.qwen3 import EagerLoRA

        self.model, self.training = model, bool(training)
        self.lora = EagerLoRA(model.lora, requires_grad=self.training)
        self._saved: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def _layers(self, x: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        m = self.model
        if _is_hybrid(m):
            return m.forward(None, mask, x=x, lora=self.lora, training=self.training)
        from graspo_b200.models.qwen3 import eager_layer, position_ids_from_mask

        pos = position_ids_from_mask(mask)
        for lw in m.layers:
            if self.training and m.gradient_checkpointing:
                x = torch.utils.checkpoint.checkpoint(eager_layer, m, lw, x, pos, mask, self.lora, True,
                                                      use_reentrant=False)
            else:
                x = eager_layer(m, lw, x, pos, mask, self.lora, self.training)
        return x

    def forward(self, mb: Microbatch) -> Microbatch:
        x_in = mb.tensors["hidden"].detach()
        if self.training:
            x_in.requires_grad_(True)
        with torch.set_grad_enabled(self.training):
            x_out = self._layers(x_in, mb.tensors["attention_mask"])
        if self.training:
            self._saved[mb.idx] = (x_in, x_out)
        mb.tensors["hidden"] = x_out.detach() if self.training else x_out
        return mb

    def backward(self, mb: Microbatch) -> Microbatch:
        x_in, x_out = self._saved.pop(mb.idx)
        if x_out.requires_grad:
            x_out.backward(mb.tensors["grad_hidden"])
        mb.tensors["grad_hidden"] = x_in.grad if x_in.grad is not None else torch.zeros_like(x_in)
        return mb

    def finish(self) -> None:
        """Add the collected LoRA gradients into ``model.lora.grads`` and start a new collection."""
        from graspo_b200.models.qwen3 import EagerLoRA

        self.lora.accumulate_grads()
        self.lora = EagerLoRA(self.model.lora, requires_grad=self.training)

    def trainable_parameters(self) -> list[torch.Tensor]:
        return [t for pair in self.lora.leaves.values() for t in pair]

    def done(self) -> None:
        self._saved.clear()


class HeadStageOp(ComputeOperator):
    def __init__(self, model, *, training: bool = True, name: str = "head") -> None:
        super().__init__(name=name, tp_size=model.ps.tp_size)
        if model.lm_head is None:
            raise ValueError("HeadStageOp needs a model stage that holds the LM head")
        self.model, self.training = model, bool(training)
        self._saved: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def _logprobs(self, hidden: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        m = self.model
        if _is_hybrid(m):
            return m.token_logprobs(hidden, targets).float()
        from graspo_b200.models.qwen3 import eager_token_logprobs

        return eager_token_logprobs(m, hidden, targets).float()

    def forward(self, mb: Microbatch) -> Microbatch:
        h = mb.tensors["hidden"].detach()
        if self.training:
            h.requires_grad_(True)
        with torch.set_grad_enabled(self.training):
            lp = self._logprobs(h[:, :-1], mb.tensors["targets"])
        if self.training:
            self._saved[mb.idx] = (h, lp)
        mb.tensors["logprobs"] = lp.detach()
        return mb

    def backward(self, mb: Microbatch) -> Microbatch:
        h, lp = self._saved.pop(mb.idx)
        lp.backward(mb.tensors["grad_logprobs"])
        mb.tensors["grad_hidden"] = h.grad
        return mb

    def done(self) -> None:
        self._saved.clear()


def build_stage_ops(model, *, training: bool = True) -> list[ComputeOperator]:
    """The operators of one model stage in order: embedding (first stage),
    decoder layers, head (last stage)."""
    ops: list[ComputeOperator] = []
    if model.embed is not None:
        ops.append(EmbedStageOp(model))
    ops.append(DecoderStageOp(model, training=training))
    if model.lm_head is not None:
        ops.append(HeadStageOp(model, training=training))
    return ops


__all__ = ["EmbedStageOp", "DecoderStageOp", "HeadStageOp", "build_stage_ops"]
