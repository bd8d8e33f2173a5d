"""Group rollout: prefill once per prompt, decode G completions per prompt.

GRASPO samples ``G`` completions of every prompt.  The reference repeats each
prompt G times and prefills all copies (reference: qwen3/adapter.py:190-230),
grows its KV cache with ``torch.cat`` every token and synchronises with the
host after every token to test for EOS (generation.py:249-276).  This engine:

* prefills each *unique* prompt once and writes its K/V into pages that the G
  rows of the group share through their block tables (prefix sharing: 1/G
  of the prompt KV memory and prefill FLOPs);
* keeps K/V in a preallocated paged pool ``[layers, pages, kv_heads, page, 128]``
  and writes each new token's K/V in place from the QK-norm/RoPE kernel;
* runs a decode step as one CUDA graph (embedding -> 36 x [norm + LoRA-down,
  QKV GEMM, QK-norm/RoPE/KV-write, paged attention, O GEMM, norm, gate/up
  GEMM with SwiGLU, down GEMM] -> LM head -> sampling + state update), with
  all per-row state (next token, cache slot, position, length, finished) on
  the device, and checks for "all rows finished" only every few steps.

The decode GEMMs are "swap-AB": weights fill the 128-row side of the
tensor-core tile and the decode batch the narrow side; the QKV / O / down
projections split K across CTAs and accumulate fp32 partial sums that the
next kernel consumes (and re-zeroes).

``EagerRolloutEngine`` is the plain-PyTorch counterpart (CPU / tests).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from graspo_b200.models.qwen3 import (
    EagerLoRA,
    Qwen3Model,
    _linear_lora,
    apply_rope,
    rmsnorm,
)
from graspo_b200.parallel.tp import copy_to_tp, reduce_from_tp


@dataclass
class RolloutResult:
    prompt_ids: torch.Tensor      # [n, P] left-padded prompts (host)
    prompt_lens: list[int]
    tokens: torch.Tensor          # [rows, max_new] generated ids (host), pad after finish
    gen_lens: list[int]           # generated tokens per row (up to and including EOS)
    group_size: int
    prefill_sec: float = 0.0
    decode_sec: float = 0.0
    decode_steps: int = 0
    splits: int = 1               # engine calls the rows were decoded in


def merge_results(parts: list[RolloutResult], pad_id: int) -> RolloutResult:
    """Concatenate the results of successive engine calls (prompt ids re-padded on the left)."""
    if len(parts) == 1:
        return parts[0]
    P = max(int(p.prompt_ids.shape[1]) for p in parts)
    ids = [torch.nn.functional.pad(p.prompt_ids, (P - p.prompt_ids.shape[1], 0), value=pad_id) for p in parts]
    return RolloutResult(
        prompt_ids=torch.cat(ids, 0), prompt_lens=[n for p in parts for n in p.prompt_lens],
        tokens=torch.cat([p.tokens for p in parts], 0), gen_lens=[n for p in parts for n in p.gen_lens],
        group_size=parts[0].group_size, prefill_sec=sum(p.prefill_sec for p in parts),
        decode_sec=sum(p.decode_sec for p in parts), decode_steps=max(p.decode_steps for p in parts),
        splits=len(parts))


def _sync(dev: torch.device) -> None:
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


def decode_attention_splits(rows: int, nkv: int, capacity: int, sms: int = 148) -> int:
    """Key-range splits so the split kernel (two resident CTAs per SM) fills the GPU
    once; each split keeps at least four 64-key tiles."""
    ctas = rows * nkv
    want = max(1, -(-2 * sms // max(ctas, 1)))
    return int(max(1, min(want, capacity // 256, 16)))


def decode_tc_splits(rows: int, nkv: int, gen_capacity: int, groups: int, prompt: int,
                     sms: int = 148) -> tuple[int, int]:
    """(row splits, prompt splits) of the tcgen05 decode attention.

    Row units (one per row, KV head and split) take at most 16 key tiles (1024
    keys) of a row's own keys and are at least two per SM; prompt units (one
    per group, KV head and split) together fill the SMs once, with at least
    four tiles each."""
    tiles = max(1, -(-gen_capacity // 64))
    units = max(1, rows * nkv)
    splits = max(-(-tiles // 16), -(-2 * sms // units))
    splits = int(max(1, min(splits, tiles, 16)))
    psplits = 1
    if prompt > 0:
        psplits = int(max(1, min(round(sms / max(1, groups * nkv)), prompt // 256, 8)))
    return splits, psplits


def swap_gemm_splits(out_features: int, rows: int, sms: int = 148, max_splits: int = 4) -> int:
    """Split-K factor for a swap-layout decode GEMM: the fewest splits that
    minimise the time of the last wave (units = 128-feature tiles x splits,
    persistent CTAs, one per SM), each split costing 1/splits of a tile."""
    tiles = -(-out_features // 128) * -(-rows // 64)
    best, best_t = 1, float("inf")
    for s in range(1, max_splits + 1):
        t = -(-tiles * s // sms) / s
        if t < best_t - 1e-9:
            best, best_t = s, t
    return best


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _gen_lengths(tokens: torch.Tensor, eos_id: int, ignore_eos: bool) -> list[int]:
    if ignore_eos:
        return [tokens.shape[1]] * tokens.shape[0]
    lens = []
    for row in tokens.tolist():
        n = len(row)
        for i, t in enumerate(row):
            if t == eos_id:
                n = i + 1
                break
        lens.append(n)
    return lens


class FusedRolloutEngine:
    def __init__(self, model: Qwen3Model, fused, *, page_size: int = 64, use_graph: bool = True,
                 graph_chunk: int = 16, fused_tp_allreduce: bool = True, comm=None) -> None:
        from graspo_b200.ops._ext import ext

        self.m = model
        self.f = fused
        self.C = ext()
        self.page = page_size
        self.use_graph = use_graph
        self.graph_chunk = graph_chunk
        self._pool_shape = None
        self.k_pool = self.v_pool = None
        self.nvtx = False  # wrap eager decode steps in NVTX ranges "decode_step"
        # tensor-parallel all-reduce of the decode loop inside the GEMM / RMSNorm
        # kernels (peer-memory tile push) instead of NCCL calls
        self.fused_tp = bool(fused_tp_allreduce) and model.ps.tp_size > 1 and model.device.type == "cuda"
        self._peer_sites: dict[tuple, object] = {}
        # pipeline parallelism: each stage runs its local layers on every step;
        # hidden states go forward by p2p, the last stage samples and broadcasts
        # the tokens to its column (no CUDA graph across the p2p boundary)
        self.comm = comm if (comm is not None and comm.active) else None
        # attend the prompt keys once per group (shared-prefix kernel).  Off by
        # default: the rows of a group run next to each other, so the prompt pages
        # they share are read from DRAM once and served from L2, and the
        # one-launch split kernel measured faster than both shared-prompt variants
        # (the mma.sync prefix + split pair and the tcgen05 kernel with prompt units)
        self.prefix_attention = False

    def _ensure_pool(self, num_pages: int) -> None:
        m = self.m
        shape = (len(m.layers), num_pages, m.nkv, self.page, m.D)
        if self._pool_shape is None or self._pool_shape[1] < num_pages:
            self.k_pool = self.v_pool = None
            if m.device.type == "cuda":
                torch.cuda.empty_cache()
            # zero-filled: slots never written (beyond a row's length) still enter
            # the tensor-core attention tiles, multiplied by zero probabilities,
            # so they must hold finite values
            self.k_pool = torch.zeros(shape, device=m.device, dtype=m.dtype)
            self.v_pool = torch.zeros(shape, device=m.device, dtype=m.dtype)
            self._pool_shape = shape

    def _vocab_gather(self, local: torch.Tensor) -> torch.Tensor:
        ps = self.m.ps
        if ps.tp_size == 1:
            return local
        parts = torch.empty((ps.tp_size, *local.shape), device=local.device, dtype=local.dtype)
        dist.all_gather_into_tensor(parts, local.contiguous(), group=ps.tp_group)
        return parts.permute(1, 0, 2).reshape(local.shape[0], -1).contiguous()

    def _lm_local(self, xn: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 logits of this rank's vocabulary shard [rows, vocab / tp]."""
        from graspo_b200.ops.gemm import gemm

        m = self.m
        if xn.shape[0] <= 128:
            return gemm(m.lm_head, xn, out, swap=True, epilogue="store_f32")
        return gemm(xn, m.lm_head, out, epilogue="store_f32")

    def _lm_logits(self, xn: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._vocab_gather(self._lm_local(xn, out))

    def _sampler_plan(self, rows: int, top_p: float) -> None:
        """Split sampler (every SM, no nucleus restriction): with a vocab-parallel
        head the shards' winners are exchanged through peer memory instead of
        gathering the logits.  Nucleus sampling keeps the single-pass sampler
        over the gathered logits."""
        m = self.m
        self._split_sample = m.device.type == "cuda" and m.include_head and top_p >= 1.0 and (
            m.ps.tp_size == 1 or self.fused_tp)
        self._sx = None
        if not self._split_sample:
            return
        want = max(1, -(-4 * 148 // max(1, rows)))
        self._samp_chunk = _round_up(-(-m.vocab_local // want), 4)
        if m.ps.tp_size > 1:
            key = ("sample", rows, 0)
            sx = self._peer_sites.get(key)
            if sx is None:
                from graspo_b200.parallel.symm import SampleExchange

                for k in [k for k in self._peer_sites if k[0] == "sample"]:
                    self._peer_sites.pop(k).close()
                sx = SampleExchange(rows, m.ps.tp_group, m.device)
                self._peer_sites[key] = sx
            self._sx = sx

    @torch.no_grad()
    def generate(
        self,
        prompts: list[list[int]],
        *,
        group_size: int,
        max_new_tokens: int,
        temperature: float,
        top_p: float,
        eos_id: int,
        pad_id: int,
        ignore_eos: bool = False,
        seed: int = 0,
        embed_hook=None,
    ) -> RolloutResult:
        """``embed_hook(ids [n, P], x [n * P, H]) -> x`` may replace prompt token
        embeddings (image features) before the prefill."""
        import time

        from graspo_b200.models.fused import AttnMeta
        from graspo_b200.ops._ext import check_errors
        from graspo_b200.ops.gemm import gemm

        m, f, C = self.m, self.f, self.C
        dev = m.device
        n, G = len(prompts), int(group_size)
        rows = n * G
        lens = [max(1, len(p)) for p in prompts]
        P = _round_up(max(lens), self.page)
        prompt_pages = P // self.page
        gen_pages = math.ceil(max_new_tokens / self.page)
        num_pages = n * prompt_pages + rows * gen_pages
        self._ensure_pool(num_pages)

        ids = torch.full((n, P), pad_id, dtype=torch.long)
        mask = torch.zeros((n, P), dtype=torch.bool)
        for i, p in enumerate(prompts):
            row = list(p) or [pad_id]
            ids[i, P - len(row):] = torch.tensor(row, dtype=torch.long)
            mask[i, P - len(row):] = True
        ids_d = ids.to(dev, non_blocking=True)
        mask_d = mask.to(dev, non_blocking=True)

        bt = torch.empty(rows, prompt_pages + gen_pages, dtype=torch.int32)
        for r in range(rows):
            i = r // G
            bt[r, :prompt_pages] = torch.arange(i * prompt_pages, (i + 1) * prompt_pages)
            base = n * prompt_pages + r * gen_pages
            bt[r, prompt_pages:] = torch.arange(base, base + gen_pages)
        bt_d = bt.to(dev)

        _sync(dev)
        t0 = time.perf_counter()
        # ---------------- prefill (unique prompts)
        meta = AttnMeta.from_mask(mask_d)
        kp, vp = self.k_pool, self.v_pool

        def sink(layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
            li = m.local_layers.index(layer_idx)
            shape = (n, prompt_pages, self.page, m.nkv, m.D)
            kp[li, : n * prompt_pages] = k.view(shape).permute(0, 1, 3, 2, 4).reshape(-1, m.nkv, self.page, m.D)
            vp[li, : n * prompt_pages] = v.view(shape).permute(0, 1, 3, 2, 4).reshape(-1, m.nkv, self.page, m.D)

        comm, ps = self.comm, m.ps
        H = m.cfg.hidden_size
        x = f.embed(ids_d) if m.include_embed else comm.recv_prev((n * P, H), torch.bfloat16)
        if embed_hook is not None and m.include_embed:
            x = embed_hook(ids_d, x)
        for lw in m.layers:
            x, _ = f.layer_forward(lw, x, meta, kv_sink=sink)
        if not m.include_head:
            comm.send_next(x)
            comm.flush()

        # ---------------- decode state
        st = {
            "next_ids": torch.zeros(rows, dtype=torch.long, device=dev),
            "slot": torch.full((rows,), P - 1, dtype=torch.long, device=dev),
            "pos": torch.tensor([lens[r // G] - 1 for r in range(rows)], dtype=torch.long, device=dev),
            "kv_len": torch.full((rows,), P, dtype=torch.int32, device=dev),
            "finished": torch.zeros(rows, dtype=torch.uint8, device=dev),
            "out": torch.full((rows, max_new_tokens), pad_id, dtype=torch.long, device=dev),
            "start": torch.tensor([P - lens[r // G] for r in range(rows)], dtype=torch.int32, device=dev),
        }
        if m.include_head:
            last = x.view(n, P, -1)[:, -1].contiguous()
            xn, _ = f.final_norm(last)
            logits_rows = self._lm_logits(xn).repeat_interleave(G, dim=0).contiguous()
            C.sample_append(logits_rows, float(temperature), float(top_p), int(seed), st["next_ids"], st["slot"],
                            st["pos"], st["kv_len"], st["finished"], st["out"], P, eos_id, pad_id, bool(ignore_eos),
                            None)
            del logits_rows, last
        self._sync_stages(st)
        del x
        _sync(dev)
        t1 = time.perf_counter()

        # ---------------- decode loop
        steps = max_new_tokens - 1
        tails = self._refresh_lora_rows()
        bufs = self._decode_buffers(rows, tails)
        bufs["qkv_u"] = bufs["qkv_ws"][:, m.q_local + 2 * m.kv_local:]
        if self.fused_tp:
            H = m.cfg.hidden_size
            self._sites = {"o": self._peer_site("o", rows, H + tails.get("w_o", 0)),
                           "d": self._peer_site("d", rows, H + tails.get("w_down", 0))}
        else:
            self._sites = {}
        cap = (prompt_pages + gen_pages) * self.page
        # shared-prefix attention: the prompt keys of a group are attended once for
        # all G rows (full tensor-core tiles), the generated keys per row
        heads_per_kv = m.nq // m.nkv
        self._prefix = (P if self.prefix_attention and dev.type == "cuda" and self.page % 64 == 0 and G > 1
                        and G * heads_per_kv <= 64 else 0)
        self._group = G
        self._prefix_splits = (max(1, min(P // 64, round(148 / max(1, n * m.nkv)))) if self._prefix else 1)
        self._splits = decode_attention_splits(rows, m.nkv, cap - self._prefix)
        slots = self._splits + (self._prefix_splits if self._prefix else 0)
        bufs["attn_scratch"] = torch.zeros(rows * m.nq * slots * (m.D + 2) + rows * m.nkv,
                                           device=dev, dtype=torch.float32)
        self._sampler_plan(rows, top_p)
        if self._split_sample:
            nch = -(-m.vocab_local // self._samp_chunk)
            bufs["samp_scratch"] = torch.zeros(rows * (1 + 2 * nch) + 2, device=dev, dtype=torch.float32)
        row_ids = torch.arange(rows, dtype=torch.long, device=dev)

        def step() -> None:
            self._decode_step(st, bufs, bt_d, row_ids, P, temperature, top_p, seed, eos_id, pad_id, ignore_eos)

        done = 0
        if steps > 0:
            if self.use_graph and dev.type == "cuda" and comm is None:
                saved = {k: v.clone() for k, v in st.items()}
                step()  # warm-up outside capture (sets kernel attributes, allocator pools)
                for k, v in saved.items():
                    st[k].copy_(v)
                for ws in ("qkv_ws", "o_ws", "d_ws"):
                    bufs[ws].zero_()
                from graspo_b200.ops._ext import launches

                graph = torch.cuda.CUDAGraph()
                before = launches.count
                with torch.cuda.graph(graph):
                    step()
                per_step = launches.count - before
                launches.count = before
                while done < steps:
                    chunk = min(self.graph_chunk, steps - done)
                    for _ in range(chunk):
                        graph.replay()
                    launches.add(per_step * chunk)
                    done += chunk
                    if not ignore_eos and bool(st["finished"].all()):
                        break
                del graph
            else:
                while done < steps:
                    if self.nvtx:
                        torch.cuda.nvtx.range_push("decode_step")
                    step()
                    if self.nvtx:
                        torch.cuda.nvtx.range_pop()
                    done += 1
                    if not ignore_eos and done % self.graph_chunk == 0 and bool(st["finished"].all()):
                        break
        if comm is not None:
            comm.broadcast_from_last(st["out"])
        _sync(dev)
        t2 = time.perf_counter()
        try:
            check_errors(dev)
        except Exception:
            # a peer wait that ran out leaves the decode sites' arrival counters
            # out of step: retire them so the next call builds zeroed ones
            for site in self._peer_sites.values():
                site.close()
            self._peer_sites.clear()
            raise
        tokens = st["out"].cpu()
        return RolloutResult(
            prompt_ids=ids, prompt_lens=lens, tokens=tokens, gen_lens=_gen_lengths(tokens, eos_id, ignore_eos),
            group_size=G, prefill_sec=t1 - t0, decode_sec=t2 - t1, decode_steps=done + 1,
        )

    def _sync_stages(self, st) -> None:
        """Pipeline: the last stage's sampled tokens (and finished flags) reach
        every stage; the other stages advance their cache bookkeeping the way
        the sampler does (slot, position and key count grow by one)."""
        if self.comm is None:
            return
        self.comm.broadcast_from_last(st["next_ids"])
        self.comm.broadcast_from_last(st["finished"])
        if not self.m.include_head:
            st["slot"] += 1
            st["pos"] += 1
            st["kv_len"].copy_(st["slot"] + 1)

    def _lora_tails(self) -> dict[str, int]:
        """Spare weight rows per projection: the width of its scaled LoRA A layout."""
        m = self.m
        if not m.layers:
            return {}
        L = m.lora.layer_layouts(m.layers[0].index, m.sizes)
        return {"w_qkv": L["a_qkv"].shape[0] if "a_qkv" in L else 0,
                "w_o": L["a_o"].shape[0] if "a_o" in L else 0,
                "w_down": L["a_down"].shape[0] if "a_down" in L else 0,
                "u_gu": L["a_gu"].shape[0] if "a_gu" in L else 0}

    def _refresh_lora_rows(self) -> dict[str, int]:
        """Write the current (scaled) LoRA A factors into the weights' spare rows."""
        m = self.m
        tails = self._lora_tails()
        m.ensure_tail_rows({k: v for k, v in tails.items() if k.startswith("w_")})
        r = m.lora.r
        self._bt = {}
        for lw in m.layers:
            L = m.lora.layer_layouts(lw.index, m.sizes)
            for name, key in (("w_qkv", "a_qkv"), ("w_o", "a_o"), ("w_down", "a_down")):
                if key in L:
                    ext = getattr(lw, f"{name}_ext")
                    ext[getattr(lw, name).shape[0]:].copy_(L[key])
            # B^T layouts for the consumer kernels' B U (rank rows contiguous over features)
            self._bt[lw.index] = {
                "qkv": L["b_qkv"][:, : 3 * r].t().contiguous() if "b_qkv" in L else None,
                "o": L["b_o"][:, :r].t().contiguous() if "b_o" in L else None,
                "down": L["b_down"][:, :r].t().contiguous() if "b_down" in L else None,
            }
        return tails

    def _peer_site(self, name: str, rows: int, width: int):
        """The fused all-reduce site ``name`` for ``rows`` x ``width`` partials (kept across calls)."""
        key = (name, rows, width)
        site = self._peer_sites.get(key)
        if site is None:
            from graspo_b200.parallel.symm import PeerReduce

            for k in [k for k in self._peer_sites if k[0] == name]:
                self._peer_sites.pop(k).close()
            site = PeerReduce(rows, width, self.m.ps.tp_group, self.m.device)
            self._peer_sites[key] = site
        return site

    def _gu_splits(self, rows: int) -> int:
        """Split-K for gate/up only when its tiles fill less than half of the
        SMs (TP >= 4 shards): the split partials' fixup through L2 measured
        slower than a partial last wave on the full-width projection."""
        if self.m.device.type != "cuda":
            return 1
        tiles = -(-2 * self.m.inter_local // 128) * -(-rows // 64)
        return swap_gemm_splits(2 * self.m.inter_local, rows) if 2 * tiles <= 148 else 1

    def _decode_buffers(self, rows: int, tails: dict[str, int]) -> dict[str, torch.Tensor]:
        m = self.m
        dev, dt = m.device, m.dtype
        H = m.cfg.hidden_size
        f32 = torch.float32
        nqkv = m.q_local + 2 * m.kv_local
        return {
            "x_a": torch.empty(rows, H, device=dev, dtype=dt),
            "x_b": torch.empty(rows, H, device=dev, dtype=dt),
            "xn": torch.empty(rows, H, device=dev, dtype=dt),
            # fp32 split-K workspaces: projection columns, then U = s A x
            "qkv_ws": torch.zeros(rows, nqkv + tails.get("w_qkv", 0), device=dev, dtype=f32),
            "q": torch.empty(rows, m.nq, m.D, device=dev, dtype=dt),
            # LoRA U columns of the q/k/v workspace (cleared after qk_norm_rope has read them)
            "qkv_u": None,
            "attn": torch.empty(rows, m.q_local, device=dev, dtype=dt),
            "o_ws": torch.zeros(rows, H + tails.get("w_o", 0), device=dev, dtype=f32),
            # U = s A xn of the gate/up LoRA (the K-extension operand of that GEMM)
            "u_gu": torch.zeros(rows, max(tails.get("u_gu", 0), 1), device=dev, dtype=dt),
            "act": torch.empty(rows, m.inter_local, device=dev, dtype=dt),
            # split-K gate/up: per-split fp32 partial tiles and per-tile arrival counters
            "gu_ws": torch.empty(self._gu_splits(rows) * rows * 2 * m.inter_local, device=dev, dtype=f32),
            "gu_ctr": torch.zeros(-(-2 * m.inter_local // 128) * -(-rows // 64), device=dev, dtype=torch.int32),
            "d_ws": torch.zeros(rows, H + tails.get("w_down", 0), device=dev, dtype=f32),
            "logits": (torch.empty(rows, m.vocab_local, device=dev, dtype=f32) if m.include_head
                       else torch.empty(0, device=dev)),
            "ones": torch.ones(H, device=dev, dtype=dt),
        }

    def _decode_step(self, st, b, bt, row_ids, P, temperature, top_p, seed, eos_id, pad_id, ignore_eos) -> None:
        """One token for every row: embedding, the decoder layers, LM head, sampling.

        LoRA: q/k/v, o and down compute U = s A x inside their base GEMM (A sits
        in spare weight rows, U lands after the projection columns of the fp32
        split-K workspace) and the consuming kernel adds B U -- qk_norm_rope
        for q/k/v, the next residual-add + RMSNorm for o and down.  gate/up
        keep the K-extension, because SwiGLU in the GEMM epilogue needs the
        complete pre-activation: the RMSNorm kernel that produces the GEMM
        input also computes its U.
        """
        from graspo_b200.ops._ext import err_word
        from graspo_b200.ops.gemm import gemm

        m, C = self.m, self.C
        eps = m.cfg.rms_norm_eps
        tp_group = m.ps.tp_group
        tp = m.ps.tp_size
        r = m.lora.r
        rows = row_ids.shape[0]
        so, sd = self._sites.get("o"), self._sites.get("d")
        # the norm kernels' bounded waits (peer sums, staged LoRA rows) report into the error word
        ew = {"err": err_word(m.device)}
        o_norm = so.norm_kwargs() if so is not None else ew
        d_norm = sd.norm_kwargs() if sd is not None else ew
        if m.include_embed:
            C.embedding(st["next_ids"], m.embed, b["x_a"])
        else:
            self.comm.recv_prev(b["x_a"].shape, b["x_a"].dtype, out=b["x_a"])
        scale = 1.0 / math.sqrt(m.D)
        b_down_prev = None
        for li, lw in enumerate(m.layers):
            L = m.lora.layer_layouts(lw.index, m.sizes)
            BT = self._bt[lw.index]
            first = li == 0
            # x_a holds the residual stream; the previous layer's down-projection
            # partial sums (d_ws, with its LoRA U) are added here, the sum stored to x_a
            C.add_rmsnorm(b["x_b"] if not first else b["x_a"], None if first else b["d_ws"],
                          None if first else b["x_a"], lw.ln1, b["xn"], None, None, None, 1.0, eps,
                          b_down_prev, r if b_down_prev is not None else 0, **({} if first else d_norm))
            has_qkv = "a_qkv" in L
            gemm(lw.w_qkv_ext if has_qkv else lw.w_qkv, b["xn"], b["qkv_ws"], swap=True, epilogue="atomic",
                 splits=3)
            C.qk_norm_rope(b["qkv_ws"], lw.q_norm, lw.k_norm, m.inv_freq, st["pos"], b["q"], self.k_pool[li],
                           self.v_pool[li], bt, row_ids, st["slot"], m.nq, m.nkv, self.page, eps,
                           BT["qkv"], r if has_qkv else 0, **ew)
            C.paged_decode_attention(b["q"], self.k_pool[li], self.v_pool[li], bt, st["start"], st["kv_len"],
                                     b["attn"], scale, self._splits, b["attn_scratch"], self._prefix, self._group,
                                     self._prefix_splits, **ew)
            has_o = "a_o" in L
            gemm(lw.w_o_ext if has_o else lw.w_o, b["attn"], b["o_ws"], swap=True, epilogue="atomic", splits=4,
                 push=so)
            if tp > 1 and so is None:
                dist.all_reduce(b["o_ws"], group=tp_group)
            a_gu = L.get("a_gu")
            ug = b["u_gu"] if a_gu is not None else None
            # only the 2r live rows of the padded A layout are dotted (the rest of U stays 0);
            # this kernel also clears the q/k/v LoRA U columns read by qk_norm_rope
            C.add_rmsnorm(b["x_a"], b["o_ws"], b["x_b"], lw.ln2, b["xn"], None,
                          a_gu[: 2 * r] if a_gu is not None else None, ug, 1.0, eps,
                          BT["o"], r if has_o else 0, **o_norm,
                          zero_tail=b["qkv_u"] if has_qkv else None)
            gu_splits = self._gu_splits(rows)
            gemm(lw.w_gu, b["xn"], b["act"], ext_ab=(L["b_gu"], ug) if a_gu is not None else None,
                 swap=True, epilogue="swiglu", splits=gu_splits,
                 aux=b["gu_ws"] if gu_splits > 1 else None, tile_ctr=b["gu_ctr"] if gu_splits > 1 else None)
            has_d = "a_down" in L
            gemm(lw.w_down_ext if has_d else lw.w_down, b["act"], b["d_ws"], swap=True, epilogue="atomic",
                 splits=4, push=sd)
            if tp > 1 and sd is None:
                dist.all_reduce(b["d_ws"], group=tp_group)
            b_down_prev = BT["down"]
        ran = len(m.layers) > 0  # a stage may hold only the LM head
        if not m.include_head:
            # stage boundary: materialise the residual stream (x_b + down output)
            # in x_a and hand it to the next stage (the norm output is unused)
            if ran:
                C.add_rmsnorm(b["x_b"], b["d_ws"], b["x_a"], b["ones"], b["xn"], None, None, None, 1.0, eps,
                              b_down_prev, r if b_down_prev is not None else 0, **d_norm)
            self.comm.send_next(b["x_a"])
            self.comm.flush()
            self._sync_stages(st)
            return
        if ran:
            C.add_rmsnorm(b["x_b"], b["d_ws"], b["x_a"], m.norm, b["xn"], None, None, None, 1.0, eps,
                          b_down_prev, r if b_down_prev is not None else 0, **d_norm)
        else:
            C.add_rmsnorm(b["x_a"], None, None, m.norm, b["xn"], None, None, None, 1.0, eps)
        if self._split_sample:
            local = self._lm_local(b["xn"], b["logits"])
            C.sample_append_split(local, float(temperature), int(seed), st["next_ids"], st["slot"], st["pos"],
                                  st["kv_len"], st["finished"], st["out"], P, eos_id, pad_id, bool(ignore_eos),
                                  m.vocab_start, b["samp_scratch"], self._samp_chunk, ew["err"],
                                  **(self._sx.kwargs() if self._sx is not None else {}))
        else:
            logits = self._lm_logits(b["xn"], b["logits"])
            C.sample_append(logits, float(temperature), float(top_p), int(seed), st["next_ids"], st["slot"],
                            st["pos"], st["kv_len"], st["finished"], st["out"], P, eos_id, pad_id, bool(ignore_eos),
                            None)
        self._sync_stages(st)


# ======================================================================= eager
class EagerRolloutEngine:
    """Plain-PyTorch rollout with a contiguous KV cache (CPU / reference path)."""

    def __init__(self, model: Qwen3Model) -> None:
        self.m = model

    def _layer(self, lw, x, pos, key_mask, cache, cur, lora):
        m = self.m
        cfg = m.cfg
        ad = m.lora
        group = m.ps.tp_group
        B, s_new, _ = x.shape
        mod = {k: ad.module(lw.index, k) for k in ("q", "k", "v", "o", "gate", "up", "down")}
        h = copy_to_tp(rmsnorm(x, lw.ln1, cfg.rms_norm_eps), group)
        q_end, k_end = m.q_local, m.q_local + m.kv_local
        q = _linear_lora(h, lw.w_qkv[:q_end], mod["q"], lora, ad.scaling, 0.0, False)
        k = _linear_lora(h, lw.w_qkv[q_end:k_end], mod["k"], lora, ad.scaling, 0.0, False)
        v = _linear_lora(h, lw.w_qkv[k_end:], mod["v"], lora, ad.scaling, 0.0, False)
        q = apply_rope(rmsnorm(q.view(B, s_new, m.nq, m.D), lw.q_norm, cfg.rms_norm_eps), pos, m.inv_freq)
        k = apply_rope(rmsnorm(k.view(B, s_new, m.nkv, m.D), lw.k_norm, cfg.rms_norm_eps), pos, m.inv_freq)
        kc, vc = cache
        kc[:, cur : cur + s_new] = k
        vc[:, cur : cur + s_new] = v.view(B, s_new, m.nkv, m.D)
        total = cur + s_new
        keys = kc[:, :total].float().transpose(1, 2).repeat_interleave(m.nq // m.nkv, 1)
        vals = vc[:, :total].float().transpose(1, 2).repeat_interleave(m.nq // m.nkv, 1)
        scores = (q.float().transpose(1, 2) @ keys.transpose(-1, -2)) / math.sqrt(m.D)
        qpos = torch.arange(cur, total, device=x.device)[:, None]
        kpos = torch.arange(total, device=x.device)[None, :]
        allowed = (kpos <= qpos)[None, None] & key_mask[:, None, None, :total]
        scores = scores.masked_fill(~allowed, float("-inf"))
        probs = torch.nan_to_num(torch.softmax(scores, -1), nan=0.0)
        attn = (probs @ vals).transpose(1, 2).reshape(B, s_new, -1).to(x.dtype)
        o = _linear_lora(attn, lw.w_o, mod["o"], lora, ad.scaling, 0.0, False)
        x = x + reduce_from_tp(o, group)
        h2 = copy_to_tp(rmsnorm(x, lw.ln2, cfg.rms_norm_eps), group)
        g = _linear_lora(h2, lw.w_gu[0::2], mod["gate"], lora, ad.scaling, 0.0, False)
        u = _linear_lora(h2, lw.w_gu[1::2], mod["up"], lora, ad.scaling, 0.0, False)
        d = _linear_lora(F.silu(g) * u, lw.w_down, mod["down"], lora, ad.scaling, 0.0, False)
        return x + reduce_from_tp(d, group)

    def _logits(self, h):
        m = self.m
        local = F.linear(rmsnorm(h, m.norm, m.cfg.rms_norm_eps).float(), m.lm_head.float())
        ps = m.ps
        if ps.tp_size > 1:
            parts = [torch.empty_like(local) for _ in range(ps.tp_size)]
            dist.all_gather(parts, local.contiguous(), group=ps.tp_group)
            local = torch.cat(parts, -1)
        return local

    @torch.no_grad()
    def generate(self, prompts, *, group_size, max_new_tokens, temperature, top_p, eos_id, pad_id,
                 ignore_eos=False, seed=0, embed_hook=None) -> RolloutResult:
        import time

        m = self.m
        dev = m.device
        n, G = len(prompts), int(group_size)
        rows = n * G
        lens = [max(1, len(p)) for p in prompts]
        P = max(lens)
        ids = torch.full((n, P), pad_id, dtype=torch.long)
        mask = torch.zeros((n, P), dtype=torch.bool)
        for i, p in enumerate(prompts):
            row = list(p) or [pad_id]
            ids[i, P - len(row):] = torch.tensor(row)
            mask[i, P - len(row):] = True
        ids_r = ids.repeat_interleave(G, 0).to(dev)
        key_mask = torch.zeros(rows, P + max_new_tokens, dtype=torch.bool, device=dev)
        key_mask[:, :P] = mask.repeat_interleave(G, 0).to(dev)
        pos = (key_mask[:, :P].long().cumsum(-1) - 1).clamp(min=0)
        caches = [
            (torch.zeros(rows, P + max_new_tokens, m.nkv, m.D, dtype=m.dtype, device=dev),
             torch.zeros(rows, P + max_new_tokens, m.nkv, m.D, dtype=m.dtype, device=dev))
            for _ in m.layers
        ]
        lora = EagerLoRA(m.lora, requires_grad=False)
        gen = torch.Generator(device="cpu").manual_seed(int(seed))
        t0 = time.perf_counter()
        x = F.embedding(ids_r, m.embed)
        if embed_hook is not None:
            xu = F.embedding(ids.to(dev), m.embed)
            xu = embed_hook(ids.to(dev), xu.reshape(-1, xu.shape[-1]).clone()).view_as(xu)
            x = xu.repeat_interleave(G, 0)
        for lw, cache in zip(m.layers, caches, strict=True):
            x = self._layer(lw, x, pos, key_mask, cache, 0, lora)
        logits = self._logits(x[:, -1])
        out = torch.full((rows, max_new_tokens), pad_id, dtype=torch.long)
        finished = torch.zeros(rows, dtype=torch.bool)
        next_pos = pos[:, -1] + 1
        t1 = time.perf_counter()
        steps = 0
        for step in range(max_new_tokens):
            tok = self._sample(logits.cpu(), temperature, top_p, gen)
            tok = torch.where(finished, torch.full_like(tok, pad_id), tok)
            if m.ps.tp_size > 1:
                tok_d = tok.to(dev)
                dist.broadcast(tok_d, src=m.ps.tp_ranks[0], group=m.ps.tp_group)
                tok = tok_d.cpu()
            out[:, step] = tok
            steps += 1
            if not ignore_eos:
                finished |= tok == eos_id
            if step == max_new_tokens - 1 or (not ignore_eos and bool(finished.all())):
                break
            key_mask[:, P + step] = True
            x = F.embedding(tok.to(dev)[:, None], m.embed)
            cur = P + step
            for lw, cache in zip(m.layers, caches, strict=True):
                x = self._layer(lw, x, next_pos[:, None], key_mask, cache, cur, lora)
            next_pos = next_pos + 1
            logits = self._logits(x[:, -1])
        t2 = time.perf_counter()
        return RolloutResult(
            prompt_ids=ids, prompt_lens=lens, tokens=out, gen_lens=_gen_lengths(out, eos_id, ignore_eos),
            group_size=G, prefill_sec=t1 - t0, decode_sec=t2 - t1, decode_steps=steps,
        )

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float, gen: torch.Generator) -> torch.Tensor:
        if temperature <= 0:
            return logits.argmax(-1)
        scaled = logits.float() / max(temperature, 1e-6)
        if 0 < top_p < 1:
            probs = torch.softmax(scaled, -1)
            sp, si = torch.sort(probs, descending=True, dim=-1)
            cum = sp.cumsum(-1)
            drop = cum - sp > top_p
            sp = sp.masked_fill(drop, 0.0)
            choice = torch.multinomial(sp / sp.sum(-1, keepdim=True), 1, generator=gen).squeeze(-1)
            return si.gather(-1, choice[:, None]).squeeze(-1)
        u = torch.rand(scaled.shape, generator=gen).clamp_(1e-20, 1 - 1e-7)
        return (scaled - torch.log(-torch.log(u))).argmax(-1)
