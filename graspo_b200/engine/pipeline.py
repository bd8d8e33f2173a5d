"""Pipeline-parallel forward / backward of the fused decoder.

A batch of rows is cut into micro-batches of ``chunk_rows`` rows.  Stage 0
embeds, every stage runs its local layers, the last stage normalises and
computes the selected-token log-probs (and the loss); hidden states travel
forward and their gradients backward between neighbouring stages over
``StageComm`` (NCCL p2p on GPUs, one stream per direction).  Every receive
is posted one receiving step ahead of the step that consumes it, so the
transfer runs under the computation before it instead of between the two.

* ``pp_logprobs``: forward only (old log-probs), GPipe order; the last stage
  broadcasts the log-probs to its pipeline column so every rank returns them
  (reference: backends/graspoflow/models/qwen35_36/logprobs.py:65-121).
* ``pp_train``: one optimizer step's forward + backward under the configured
  schedule (``one_f_one_b`` by default: warm-up forwards, then alternating
  forward / backward, then the drain -- parallel/schedule.py).  The loss of a
  micro-batch is weighted by its share of the rows, so the accumulated
  gradient equals the unchunked one (reference: training.py:727-1043).
  Backward recomputes each stage's layers from their saved inputs.
"""

from __future__ import annotations

from typing import Callable

import torch

from graspo_b200.models.fused import AttnMeta, FusedQwen3
from graspo_b200.ops._ext import ext
from graspo_b200.parallel.p2p import StageComm
from graspo_b200.parallel.schedule import PipelineAction, get_scheduler, peak_inflight
from graspo_b200.utils.timing import NULL_CLOCK, PhaseClock, schedule_phases

# the fused layers produce bf16 activations (the GEMMs store bf16); stage
# transfers use it on the wire whatever the model's parameter dtype
ACT_DTYPE = torch.bfloat16


def _chunks(B: int, rows: int) -> list[slice]:
    rows = max(1, int(rows))
    return [slice(i, min(B, i + rows)) for i in range(0, B, rows)]


def _sp_pad(f: FusedQwen3, seq, mask, targets):
    """Under sequence parallelism every micro-batch's tokens split evenly over the
    TP ranks: pad the sequence dimension to a multiple of TP with masked pad
    tokens.  Returns the padded seq, mask and targets and the token divisor
    (``tp`` with SP, else 1)."""
    tp = f.m.ps.tp_size if f.sp else 1
    pad = (-seq.shape[1]) % tp
    if pad:
        seq = torch.cat([seq, seq.new_zeros(seq.shape[0], pad)], 1)
        mask = torch.cat([mask, mask.new_zeros(mask.shape[0], pad)], 1)
        targets = torch.cat([targets, targets.new_zeros(targets.shape[0], pad)], 1)
    return seq, mask, targets, tp


def _full_targets(tgt: torch.Tensor) -> torch.Tensor:
    B, S1 = tgt.shape
    full = torch.zeros(B, S1 + 1, dtype=torch.long, device=tgt.device)
    full[:, :-1] = tgt
    return full


class _RecvAhead:
    """Posts every step's receive one receiving step early.

    ``needs[k]`` is the receive of plan step ``k``: ("prev", shape) for a
    forward step past the first stage, ("next", shape) for a backward step
    before the last, or None.  ``advance(k)``, called as step ``k`` starts,
    posts in plan order every receive up to the first receiving step after
    ``k``, so that step's transfer runs while step ``k`` computes.  Plan order
    is the order the neighbour sends in (forward micro-batches ascending,
    backward micro-batches ascending), which keeps each direction's queue
    matched."""

    def __init__(self, comm: StageComm, needs: list, dtype: torch.dtype) -> None:
        self.comm, self.dtype = comm, dtype
        self.order = [(k, n) for k, n in enumerate(needs) if n is not None]
        self.posted = 0

    def advance(self, k: int) -> None:
        last = next((i for i, (step, _) in enumerate(self.order) if step > k), len(self.order) - 1)
        while self.posted <= last:
            side, shape = self.order[self.posted][1]
            (self.comm.prefetch_prev if side == "prev" else self.comm.prefetch_next)(shape, self.dtype)
            self.posted += 1


def _plan_needs(plan, chunks: list[slice], ps, shape_of) -> list:
    needs = []
    for _, step in plan:
        rows = chunks[step.microbatch_idx].stop - chunks[step.microbatch_idx].start
        if step.action == PipelineAction.FORWARD:
            needs.append(None if ps.is_first_stage else ("prev", shape_of(rows)))
        else:
            needs.append(None if ps.is_last_stage else ("next", shape_of(rows)))
    return needs


def pp_logprobs(f: FusedQwen3, comm: StageComm, seq: torch.Tensor, mask: torch.Tensor,
                targets: torch.Tensor, *, chunk_rows: int, embed_hook=None) -> torch.Tensor:
    """log p(targets) [B, S-1] on every stage of the column (forward only).

    With sequence parallelism each TP rank carries, and sends to the same TP
    rank of the next stage, its 1/tp share of a micro-batch's tokens.
    ``embed_hook`` (image inputs) edits the first stage's embeddings, one
    micro-batch's rows at a time."""
    m, ps = f.m, comm.ps
    B, S_in = seq.shape
    seq, mask, targets, tp = _sp_pad(f, seq, mask, targets)
    S = seq.shape[1]
    H = m.cfg.hidden_size
    full = _full_targets(targets)
    outs = []
    chunks = _chunks(B, chunk_rows)
    hooks = embed_hook.split_rows(seq, chunks) if embed_hook is not None and ps.is_first_stage else None
    ahead = _RecvAhead(comm, [None if ps.is_first_stage else ("prev", ((c.stop - c.start) * S // tp, H))
                              for c in chunks], ACT_DTYPE)
    for k, sl in enumerate(chunks):
        rows = sl.stop - sl.start
        ahead.advance(k)
        meta = AttnMeta.from_mask(mask[sl])
        if ps.is_first_stage:
            x = f.embed(seq[sl])
            x = f.sp_shard(hooks[k](seq[sl], x).detach() if hooks is not None else x)
        else:
            x = comm.recv_prev((rows * S // tp, H), ACT_DTYPE)
        xL, _ = f.stage_forward(x, meta)
        if ps.is_last_stage:
            hn, _ = f.final_norm(xL)
            lp, _ = f.token_logprobs(f.sp_gather(hn), full[sl].reshape(-1))
            outs.append(lp.view(rows, S)[:, : S_in - 1])
        else:
            comm.send_next(xL.to(ACT_DTYPE))
    comm.flush()
    logp = torch.cat(outs, 0).contiguous() if ps.is_last_stage else torch.empty(B, S_in - 1, device=seq.device)
    return comm.broadcast_from_last(logp)


LossFn = Callable[[torch.Tensor, slice], tuple[torch.Tensor, torch.Tensor]]


def pp_train(f: FusedQwen3, comm: StageComm, seq: torch.Tensor, mask: torch.Tensor, targets: torch.Tensor,
             loss_fn: LossFn, *, seed: int, chunk_rows: int, schedule: str = "one_f_one_b",
             clock: PhaseClock = NULL_CLOCK, embed_hook=None, max_inflight: int = 0) -> torch.Tensor:
    """Forward + backward of one optimizer step into the LoRA gradient buffer.

    ``loss_fn(logp_chunk [rows, S-1], row_slice)`` runs on the last stage and
    returns (loss contribution [1], d loss / d logp_chunk); contributions must
    already carry the chunk's weight.  Returns the summed loss on every stage.
    ``clock`` collects the stage timers (recv / send / compute / head / loss /
    backward, and the fill / steady / drain phases of the schedule).
    ``max_inflight`` > 0 caps the micro-batches a stage holds activations for
    (``graspoflow.pp_max_inflight_microbatches``).
    ``embed_hook`` (image inputs) edits the first stage's embeddings per
    micro-batch; with LoRA on the vision tower, the embedding gradient of
    each micro-batch's image rows is collected and sent through the tower
    once, after the last backward.
    """
    m, ps = f.m, comm.ps
    C = ext()
    B, S_in = seq.shape
    seq, mask, targets, tp = _sp_pad(f, seq, mask, targets)
    S = seq.shape[1]
    H = m.cfg.hidden_size
    full = _full_targets(targets)
    chunks = _chunks(B, chunk_rows)
    plan = schedule_phases(get_scheduler(schedule, pp_size=ps.pp_size, pp_rank=ps.pp_rank), len(chunks),
                           max_inflight)
    clock.peak("pipeline_chunks_per_optimizer_step", len(chunks))
    clock.peak("pipeline_peak_inflight_microbatches", peak_inflight([st for _, st in plan]))
    ahead = _RecvAhead(comm, _plan_needs(plan, chunks, ps, lambda rows: (rows * S // tp, H)), ACT_DTYPE)
    hooks = embed_hook.split_rows(seq, chunks) if embed_hook is not None and ps.is_first_stage else None
    graphs: dict[int, torch.Tensor] = {}  # micro-batch -> embeddings carrying the image-feature graph
    saved: dict[int, tuple] = {}
    total = torch.zeros(1, device=seq.device, dtype=torch.float32)
    for k, (phase, step) in enumerate(plan):
        t_step = clock.now()
        c = step.microbatch_idx
        sl = chunks[c]
        rows = sl.stop - sl.start
        ahead.advance(k)
        if step.action == PipelineAction.FORWARD:
            meta = AttnMeta.from_mask(mask[sl])
            if ps.is_first_stage:
                x = f.embed(seq[sl])
                if hooks is not None:
                    x = hooks[c](seq[sl], x)
                    if x.requires_grad:
                        graphs[c], x = x, x.detach()
                x = f.sp_shard(x)
            else:
                with clock.time("pipeline_recv_sec"):
                    x = comm.recv_prev((rows * S // tp, H), ACT_DTYPE)
            with clock.time("pipeline_stage_compute_sec"):
                xL, inputs = f.stage_forward(x, meta, train=True, seed=seed, keep_inputs=True)
            clock.calls["pipeline_forward_calls"] += 1
            if ps.is_last_stage:
                with clock.time("pipeline_lm_head_sec"):
                    hn, rstd = f.final_norm(xL)
                    hn = f.sp_gather(hn)
                    fc = full[sl].reshape(-1).contiguous()
                    lp, lse = f.token_logprobs(hn, fc)
                with clock.time("pipeline_loss_sec"):
                    loss_c, dlogp = loss_fn(lp.view(rows, S)[:, : S_in - 1], sl)
                    total += loss_c.reshape(1)
                saved[c] = (meta, inputs, xL, hn, rstd, fc, lse, dlogp)
            else:
                with clock.time("pipeline_send_sec"):
                    comm.send_next(xL.to(ACT_DTYPE))
                saved[c] = (meta, inputs)
        else:
            if ps.is_last_stage:
                meta, inputs, xL, hn, rstd, fc, lse, dlogp = saved.pop(c)
                with clock.time("pipeline_backward_autograd_sec"):
                    g = torch.zeros(rows, S, device=seq.device, dtype=torch.float32)
                    g[:, : S_in - 1] = dlogp
                    # the head's input gradient, this rank's token shard under SP
                    dhn = f.token_logprobs_backward(hn, fc, lse, g.view(-1))
                    dx = torch.empty_like(xL)
                    C.rmsnorm_bwd(dhn, xL, m.norm, rstd, None, dx, m.cfg.rms_norm_eps)
                del dhn, hn, xL
            else:
                meta, inputs = saved.pop(c)
                with clock.time("pipeline_grad_recv_sec"):
                    dx = comm.recv_next((rows * S // tp, H), ACT_DTYPE)
            with clock.time("pipeline_backward_autograd_sec"):
                dx_in = f.stage_backward(inputs, dx, meta, train=True, seed=seed)
                g0 = graphs.pop(c, None)
                if g0 is not None:
                    torch.autograd.backward(g0, f.sp_gather(dx_in).view_as(g0).to(g0.dtype))
            if not ps.is_first_stage:
                with clock.time("pipeline_grad_send_sec"):
                    comm.send_prev(dx_in.to(ACT_DTYPE))
        clock.add(f"{phase}_sec", clock.now() - t_step)
    comm.flush()
    if hooks is not None:
        embed_hook.backward_into_tower()
    return comm.broadcast_from_last(total)


def _mrope(model, seq, mask, hook):
    """Multimodal positions of a micro-batch with images (every stage needs them)."""
    if hook is None or not hook.grids or not hasattr(model, "mrope_positions"):
        return None
    return model.mrope_positions(seq, mask, hook)


# ---------------------------------------------------------------- autograd stages
# Families without the fused kernel path (the Qwen3.5 hybrid) pipeline their
# autograd forward instead: a stage runs ``model.forward(..., x=<previous
# stage output>)`` with per-layer gradient checkpointing, the last stage turns
# the hidden states into log-probs and the micro-batch loss, and the backward of
# a micro-batch is one ``backward`` call whose input gradient goes upstream.
# Same chunking, schedules and transfers as the fused functions above
# (reference: models/qwen35_36/training.py:567-1043, logprobs.py:65-121).


def pp_logprobs_autograd(model, comm: StageComm, seq: torch.Tensor, mask: torch.Tensor, targets: torch.Tensor, *,
                         chunk_rows: int, embed_hook=None) -> torch.Tensor:
    """log p(targets) [B, S-1] on every stage of the column (forward only).

    With ``embed_hook`` (image inputs) the first stage places the image
    features and every stage uses the multimodal positions of its micro-batch."""
    from graspo_b200.models.qwen3 import EagerLoRA

    ps = comm.ps
    B, S = seq.shape
    H = model.cfg.hidden_size
    outs = []
    lora = EagerLoRA(model.lora, requires_grad=False)
    chunks = _chunks(B, chunk_rows)
    hooks = embed_hook.split_rows(seq, chunks) if embed_hook is not None else [None] * len(chunks)
    ahead = _RecvAhead(comm, [None if ps.is_first_stage else ("prev", (c.stop - c.start, S, H))
                              for c in chunks], model.dtype)
    with torch.no_grad():
        for k, sl in enumerate(chunks):
            rows = sl.stop - sl.start
            ahead.advance(k)
            x = None if ps.is_first_stage else comm.recv_prev((rows, S, H), model.dtype)
            xL = model.forward(seq[sl], mask[sl], x=x, lora=lora, pos=_mrope(model, seq[sl], mask[sl], hooks[k]),
                               embed_hook=hooks[k] if ps.is_first_stage else None)
            if ps.is_last_stage:
                outs.append(model.token_logprobs(xL[:, :-1], targets[sl]).float())
            else:
                comm.send_next(xL)
    comm.flush()
    logp = torch.cat(outs, 0).contiguous() if ps.is_last_stage else \
        torch.empty(B, S - 1, device=seq.device, dtype=torch.float32)
    return comm.broadcast_from_last(logp)


def pp_train_autograd(model, comm: StageComm, seq: torch.Tensor, mask: torch.Tensor, targets: torch.Tensor,
                      loss_fn: Callable[[torch.Tensor, slice], torch.Tensor], *, chunk_rows: int,
                      schedule: str = "one_f_one_b", clock: PhaseClock = NULL_CLOCK,
                      embed_hook=None, max_inflight: int = 0) -> torch.Tensor:
    """Forward + backward of one optimizer step into ``model.lora.grads``.

    ``loss_fn(logp_chunk [rows, S-1], row_slice)`` runs on the last stage and
    returns the chunk's differentiable loss, already weighted by its share.
    Returns the summed loss on every stage."""
    from graspo_b200.models.qwen3 import EagerLoRA

    ps = comm.ps
    B, S = seq.shape
    H = model.cfg.hidden_size
    chunks = _chunks(B, chunk_rows)
    plan = schedule_phases(get_scheduler(schedule, pp_size=ps.pp_size, pp_rank=ps.pp_rank), len(chunks),
                           max_inflight)
    clock.peak("pipeline_chunks_per_optimizer_step", len(chunks))
    clock.peak("pipeline_peak_inflight_microbatches", peak_inflight([st for _, st in plan]))
    lora = EagerLoRA(model.lora, requires_grad=True)
    ahead = _RecvAhead(comm, _plan_needs(plan, chunks, ps, lambda rows: (rows, S, H)), model.dtype)
    hooks = embed_hook.split_rows(seq, chunks) if embed_hook is not None else [None] * len(chunks)
    saved: dict[int, tuple] = {}
    total = torch.zeros(1, device=seq.device, dtype=torch.float32)
    for k, (phase, step) in enumerate(plan):
        t_step = clock.now()
        c = step.microbatch_idx
        sl = chunks[c]
        rows = sl.stop - sl.start
        ahead.advance(k)
        if step.action == PipelineAction.FORWARD:
            x = None
            if not ps.is_first_stage:
                with clock.time("pipeline_recv_sec"):
                    x = comm.recv_prev((rows, S, H), model.dtype).requires_grad_(True)
            with torch.enable_grad():
                with clock.time("pipeline_stage_compute_sec"):
                    xL = model.forward(seq[sl], mask[sl], x=x, lora=lora, training=True,
                                       pos=_mrope(model, seq[sl], mask[sl], hooks[c]),
                                       embed_hook=hooks[c] if ps.is_first_stage else None)
                clock.calls["pipeline_forward_calls"] += 1
                if ps.is_last_stage:
                    with clock.time("pipeline_lm_head_sec"):
                        lp = model.token_logprobs(xL[:, :-1], targets[sl]).float()
                    with clock.time("pipeline_loss_sec"):
                        out = loss_fn(lp, sl).reshape(1)
                        total += out.detach()
                else:
                    with clock.time("pipeline_send_sec"):
                        comm.send_next(xL.detach())
                    out = xL
            saved[c] = (x, out)
        else:
            x, out = saved.pop(c)
            grad = None
            if not ps.is_last_stage:
                with clock.time("pipeline_grad_recv_sec"):
                    grad = comm.recv_next((rows, S, H), model.dtype)
            with clock.time("pipeline_backward_autograd_sec"):
                if out.requires_grad:
                    out.backward(grad)
            if not ps.is_first_stage:
                with clock.time("pipeline_grad_send_sec"):
                    comm.send_prev(x.grad if x.grad is not None else torch.zeros_like(x))
        clock.add(f"{phase}_sec", clock.now() - t_step)
    comm.flush()
    lora.accumulate_grads()
    if embed_hook is not None:
        embed_hook.backward_into_tower()
    return comm.broadcast_from_last(total)
