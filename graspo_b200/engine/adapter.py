"""Qwen3 adapter: model setup, rollout, log-probs, GRASPO/SFT optimisation, checkpoints.

One adapter per rank.  ``setup()`` initialises the TP x PP x DP process
groups, the tokenizer, the model shard (with LoRA targets resolved against the
family's canonical names, an optional PEFT warm start) and the optimizer.
Execution is the fused sm_100a path on a GPU (``graspoflow.kernel_backend:
fused``) and the plain-PyTorch path otherwise (CPU / gloo, or ``eager``).

Optimisation semantics follow the reference (qwen3/adapter.py:367-476,
qwen35_36/training.py:352-481): ``optimize_iterations_per_step`` passes over
the replay data in a seeded shuffle, micro-batches of
``optimize_prompt_batch_size`` completions, one clipped AdamW step per
micro-batch, a step is skipped when the loss or gradient norm is not finite.
Differences: the shuffle is computed identically on every rank instead of
being broadcast; data-parallel replicas average their LoRA gradients before
each step; the global gradient norm spans all TP/PP ranks; TP input
gradients of column-parallel projections are all-reduced.
"""

from __future__ import annotations

import json
import logging
import math
import os
import random
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from graspo_b200.core.buffer import Experience
from graspo_b200.core.chat_template import render_messages
from graspo_b200.core.completion import ParsedCompletion
from graspo_b200.core.lora_targets import resolve_lora_target_modules
from graspo_b200.core.loss import GRASPOLoss
from graspo_b200.core.tool_parser import parse_qwen_tool_completion
from graspo_b200.engine.optim import FlatAdamW, lr_lambda
from graspo_b200.engine.runtime import NativeGeneration
from graspo_b200.models.config import load_decoder_config, lora_available_targets
from graspo_b200.models.loader import SafetensorIndex
from graspo_b200.models.qwen3 import EagerLoRA, Qwen3Model, eager_stage_forward, eager_token_logprobs
from graspo_b200.parallel import state as pstate
from graspo_b200.parallel.placement import build_placement_plan, placement_summary
from graspo_b200.utils.timing import NULL_CLOCK

log = logging.getLogger("graspo.adapter")


def _dtype(name: str) -> torch.dtype:
    n = str(name).lower()
    return {"bf16": torch.bfloat16, "bfloat16": torch.bfloat16, "fp16": torch.float16, "float16": torch.float16,
            "fp32": torch.float32, "float32": torch.float32}[n]


def collate(items: list[Experience], device: torch.device, pad_id: int):
    """Right-pad experiences to a common length and move them to ``device``."""
    S = max(int(e.sequences.shape[0]) for e in items)
    B = len(items)
    seq = torch.full((B, S), pad_id, dtype=torch.long)
    att = torch.zeros((B, S), dtype=torch.bool)
    old = torch.zeros((B, S - 1), dtype=torch.float32)
    adv = torch.zeros((B, S - 1), dtype=torch.float32)
    act = torch.zeros((B, S - 1), dtype=torch.bool)
    for i, e in enumerate(items):
        n = int(e.sequences.shape[0])
        seq[i, :n] = e.sequences
        att[i, :n] = e.attention_mask.bool()
        old[i, : n - 1] = e.old_log_probs
        adv[i, : n - 1] = e.advantages
        act[i, : n - 1] = e.action_mask.bool()
    pin = device.type == "cuda"
    move = (lambda t: t.pin_memory().to(device, non_blocking=True)) if pin else (lambda t: t.to(device))
    return move(seq), move(att), move(old), move(adv), move(act)


class Qwen3Adapter:
    families: tuple[str, ...] = ("qwen3",)
    model_class = Qwen3Model
    # pipeline stages through the autograd forward (families without the fused path)
    autograd_pipeline = False
    # phase clock of the running train_batch call (no timing outside one)
    _clock = NULL_CLOCK

    def __new__(cls, config: Any = None, *args: Any, **kwargs: Any):
        # the default adapter serves both families: a qwen3_5 checkpoint gets the hybrid adapter
        if cls is Qwen3Adapter and config is not None:
            try:
                family = load_decoder_config(Path(config.model.model_path)).family
            except (OSError, ValueError, KeyError, AttributeError):
                family = None
            if family == "qwen3_5_text":
                cls = Qwen35Adapter
        return super().__new__(cls)

    completion_parser_name = "qwen_tool_call"

    def __init__(self, config: Any) -> None:
        self.config = config
        self.ps: pstate.ParallelState | None = None
        self.model: Qwen3Model | None = None
        self.tokenizer = None
        self.optimizer: FlatAdamW | None = None
        self.placement = None
        self._train_batch_call_index = 0
        self.loss_fn = GRASPOLoss(config.training.policy_ratio_clip_eps)

    # ------------------------------------------------------------ properties
    @property
    def rank(self) -> int:
        return self.ps.rank if self.ps else 0

    @property
    def tp_rank(self) -> int:
        return self.ps.tp_rank if self.ps else 0

    @property
    def device(self) -> torch.device:
        return self.ps.device if self.ps else torch.device("cpu")

    @property
    def fused(self) -> bool:
        return self.device.type == "cuda" and self.config.graspoflow.kernel_backend == "fused"

    def is_primary(self) -> bool:
        return self.rank == 0

    # ------------------------------------------------------------ setup
    def setup(self) -> None:
        cfg = self.config
        flow = cfg.graspoflow
        self.ps = pstate.initialize(flow.tp_size, flow.pp_size, flow.dp_size, timeout_sec=flow.pg_timeout_sec)
        from graspo_b200.parallel.p2p import StageComm

        self._comm = StageComm(self.ps)
        if self.ps.pp_size > 1 and not (self.fused or self.autograd_pipeline):
            raise NotImplementedError("pipeline parallelism of this family runs on the fused sm_100a kernels (GPUs)")
        model_path = Path(cfg.model.model_path)
        if not model_path.exists():
            raise FileNotFoundError(f"model.model_path does not exist: {model_path}")
        from graspo_b200.utils.tokenizer import load_tokenizer

        self.tokenizer = load_tokenizer(model_path)
        hf = load_decoder_config(model_path)
        if hf.family not in self.families:
            raise ValueError(f"{type(self).__name__} serves the {'/'.join(self.families)} family; got {hf.family}")
        targets = resolve_lora_target_modules(
            cfg.lora.target_modules or (cfg.lora.target_preset,), available=lora_available_targets(hf)
        )
        self.placement = build_placement_plan(
            strategy=flow.placement_strategy, model_family=hf.family, num_hidden_layers=hf.num_hidden_layers,
            tp_size=self.ps.tp_size, pp_size=self.ps.pp_size, tp_rank=self.ps.tp_rank, pp_rank=self.ps.pp_rank,
            layer_types=hf.layer_types, manual_ranges=flow.layer_ranges,
        )
        dtype = _dtype(cfg.model.torch_dtype)
        if self.device.type == "cpu" and dtype != torch.float32:
            dtype = torch.float32
        loader = SafetensorIndex(model_path)
        self.model = self.model_class(
            hf, loader, ps=self.ps, local_layers=list(self.placement.local_layer_indices),
            include_embed=self.placement.include_embeddings, include_head=self.placement.include_lm_head,
            lora_targets=set(targets.resolved), lora_r=cfg.lora.r, lora_alpha=cfg.lora.alpha,
            lora_dropout=cfg.lora.dropout, dtype=dtype, device=self.device, seed=cfg.training.seed,
            gradient_checkpointing=cfg.model.gradient_checkpointing,
        )
        loader.close()
        enabled = set(self.model.enabled_lora_target_names())
        if self.ps.pp_size > 1 and self.ps.distributed:
            # a stage holds some layer kinds only: the targets must be covered by the whole pipeline
            parts: list = [None] * self.ps.pp_size
            dist.all_gather_object(parts, sorted(enabled), group=self.ps.pp_group)
            enabled = set().union(*map(set, parts))
        missing = sorted(set(targets.resolved) - enabled)
        if missing:
            raise ValueError("Resolved LoRA target(s) are not implemented by this model: " + ", ".join(missing))
        if cfg.lora.adapter_path:
            from graspo_b200.models.lora_io import load_peft_adapter

            load_peft_adapter(self.model, cfg.lora.adapter_path)
        self._build_optimizer()
        self._engine = None
        self._fused = None
        if self.fused:
            from graspo_b200.engine.rollout import FusedRolloutEngine
            from graspo_b200.models.fused import FusedQwen3

            # training / log-prob passes (optionally sequence-parallel); the rollout
            # engine keeps whole-sequence prefill
            self._fused = FusedQwen3(self.model, sequence_parallel=flow.sequence_parallel)
            self._engine = FusedRolloutEngine(self.model, FusedQwen3(self.model), page_size=flow.kv_page_size,
                                              use_graph=flow.cuda_graph_decode,
                                              fused_tp_allreduce=flow.decode_tp_allreduce == "fused",
                                              comm=self._comm)
        else:
            self._engine = self._eager_engine()
        self._print_rank0({
            "event": "adapter_ready", "rank": self.rank, "tp_rank": self.tp_rank, "tp_size": self.ps.tp_size,
            "dp_size": self.ps.dp_size, "pp_size": self.ps.pp_size, "backend": "fused" if self.fused else "eager",
            "trainable_parameters_local": int(self.model.lora.numel),
            "lora_target_modules": sorted(targets.resolved),
            "lora_target_signature": self.model.lora_target_signature(),
            "placement": placement_summary(self.placement),
        })

    def _eager_engine(self):
        from graspo_b200.engine.rollout import EagerRolloutEngine

        return EagerRolloutEngine(self.model)

    def _build_optimizer(self) -> None:
        tr = self.config.training
        sched = tr.lr_scheduler
        fn = None
        if sched.type != "constant":
            if int(tr.max_steps) <= 0:
                raise ValueError("lr_scheduler.type other than constant requires training.max_steps > 0")
            total = int(tr.max_steps) * int(tr.optimize_iterations_per_step) * int(tr.rollout_group_size)
            if total <= int(sched.warmup_steps):
                raise ValueError(f"lr_scheduler: total steps ({total}) must exceed warmup_steps ({sched.warmup_steps})")
            fn = lr_lambda(sched.type, int(sched.warmup_steps), total, float(sched.min_lr_ratio))
        self.optimizer = FlatAdamW(self.model.lora, lr=tr.learning_rate, weight_decay=tr.weight_decay,
                                   schedule=fn, ps=self.ps)
        if not self.config.graspoflow.use_kv_cache_for_rollout:
            log.warning("graspoflow.use_kv_cache_for_rollout=false: rollouts always decode from the paged KV "
                        "cache here (recomputing the whole prefix for every token is not implemented)")
        self._rank_event("setup_after")

    def _print_rank0(self, payload: dict) -> None:
        if self.rank == 0:
            print(json.dumps(payload, ensure_ascii=False, default=str), flush=True)

    # ------------------------------------------------------------ prompts
    def format_messages(self, messages, chat_template_kwargs=None, *, tools=None) -> str:
        return render_messages(self.tokenizer, messages, chat_template_kwargs, tools=tools)

    def encode_prompts(self, message_batches, tool_batches, max_prompt_length, chat_template_kwargs) -> list[list[int]]:
        tool_batches = tool_batches or [None] * len(message_batches)
        texts = [self.format_messages(msgs, chat_template_kwargs, tools=tools)
                 for msgs, tools in zip(message_batches, tool_batches, strict=True)]
        enc = self.tokenizer(texts, truncation=True, max_length=int(max_prompt_length), padding=False,
                             add_special_tokens=False)
        return [list(ids) for ids in enc["input_ids"]]

    # ------------------------------------------------------------ rollout
    def generate_from_token_ids(self, prompts: list[list[int]], *, rollout_group_size: int, max_new_tokens: int,
                                temperature: float, top_p: float, seed: int | None = None):
        tok = self.tokenizer
        eos = int(tok.eos_token_id)
        pad = int(tok.pad_token_id if tok.pad_token_id is not None else eos)
        flow = self.config.graspoflow
        seed = int(self.config.training.seed) * 1_000_003 + self._train_batch_call_index if seed is None else seed
        # every TP rank must draw the same tokens: derive the seed from the DP replica only
        seed += 7919 * (self.ps.dp_rank if self.ps else 0)
        # graspoflow.rollout_engine_batch bounds the rows decoded together (0: all at once)
        limit = int(flow.rollout_engine_batch)
        per = max(1, limit // max(1, rollout_group_size)) if limit > 0 else max(1, len(prompts))
        parts = []
        for ci, start in enumerate(range(0, len(prompts), per)):
            parts.append(self._engine.generate(
                prompts[start : start + per], group_size=rollout_group_size, max_new_tokens=max_new_tokens,
                temperature=temperature, top_p=top_p, eos_id=eos, pad_id=pad,
                ignore_eos=bool(flow.benchmark_ignore_eos), seed=seed + 104729 * ci))
            if flow.empty_cache_after_rollout_split and self.device.type == "cuda":
                torch.cuda.empty_cache()
        from graspo_b200.engine.rollout import merge_results

        return merge_results(parts, pad)

    def generate_groups(self, *, message_batches=None, tool_batches=None, rollout_group_size: int,
                        max_new_tokens: int, max_prompt_length: int | None = None, temperature: float = 1.0,
                        top_p: float = 1.0, chat_template_kwargs: dict | None = None, **_: Any) -> list[NativeGeneration]:
        if not message_batches:
            return []
        t0 = time.monotonic()
        max_len = int(max_prompt_length or self.config.data.max_prompt_length)
        prompts = self.encode_prompts(message_batches, tool_batches, max_len, chat_template_kwargs)
        tokenize_sec = time.monotonic() - t0
        res = self.generate_from_token_ids(prompts, rollout_group_size=rollout_group_size,
                                           max_new_tokens=max_new_tokens, temperature=temperature, top_p=top_p)
        return self._generations(res, tokenize_sec, time.monotonic() - t0)

    def generate_sample_groups(self, *, samples: list[Any], **kwargs: Any) -> list[NativeGeneration]:
        self._rank_event("rollout_before", {"samples": len(samples)})
        if any(getattr(s, "media", None) for s in samples):
            out = self._generate_multimodal(samples, **kwargs)
        else:
            out = self.generate_groups(message_batches=[s.messages for s in samples],
                                       tool_batches=[s.tools for s in samples], **kwargs)
        self._rank_event("rollout_after", {"groups": len(out)})
        return out

    # ------------------------------------------------------------ images
    @property
    def _vision_pad_id(self) -> int:
        """The image placeholder token: config.json ``image_token_id`` (the Qwen-VL
        chat templates write ``<|image_pad|>``), else the tokenizer's own."""
        tid = (getattr(self.model.cfg, "extra", None) or {}).get("image_token_id")
        if tid is not None:
            return int(tid)
        unk = getattr(self.tokenizer, "unk_token_id", None)
        for name in ("<|image_pad|>", "<|vision_pad|>"):
            i = self.tokenizer.convert_tokens_to_ids(name)
            if i is not None and i != unk:
                return int(i)
        raise ValueError("no image placeholder token (config.json image_token_id)")

    def _sft_images(self, item: dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor, list[dict]]:
        """An SFT item's ids and labels with each image placeholder repeated once per
        merged vision token (labels -100 there), and the item's images."""
        from graspo_b200.models.vision import expand_image_placeholders, image_grid, image_size, merged_tokens

        row = item.get("_multimodal_row")
        vc = getattr(self.model, "vision_cfg", None)
        if not row or vc is None:
            return item["input_ids"], item["labels"], []
        media = [m for m in row.get("media") or [] if m.get("type") == "image"]
        if len(media) != len(row.get("media") or []):
            raise NotImplementedError("video inputs are not supported")
        pad = self._vision_pad_id
        counts = [merged_tokens(image_grid(*image_size(m["path"]), vc), vc) for m in media]
        ids = item["input_ids"].tolist()
        labels = item["labels"].tolist()
        out_ids = expand_image_placeholders(ids, pad, counts)
        out_labels, k = [], 0
        for t, lab in zip(ids, labels, strict=True):
            if t == pad and k < len(counts):
                out_labels.extend([-100] * counts[k])
                k += 1
            else:
                out_labels.append(lab)
        return torch.tensor(out_ids), torch.tensor(out_labels), media

    def _image_features(self, media_rows: list[list[dict]], vision_lora=None):
        """Vision-tower features of every image of every row, rows in order, and
        the merged grid of each image.  Features are cached per image path while
        the tower is frozen; with vision LoRA targets they follow the current
        factors (``vision_lora``: the pass's LoRA leaves, with gradients when training).

        Video inputs are rejected, as in the reference, whose data path blocks
        them (src/graspo/backends/graspoflow/multimodal.py:224, 253)."""
        from graspo_b200.models.vision import VisionLoRA, load_image, preprocess

        vt = getattr(self.model, "vision", None)
        if vt is None:
            raise NotImplementedError("this checkpoint has no vision tower (config.json vision_config)")
        if vision_lora is None and self.model.lora.vision_modules():
            vision_lora = VisionLoRA(self.model.lora, training=False)
        cache = self.__dict__.setdefault("_image_cache", {})
        if len(cache) > 512 or vision_lora is not None:
            cache.clear()
        feats, grids = [], []
        m = vt.cfg.spatial_merge_size
        for media in media_rows:
            for item in media or []:
                if item.get("type") != "image":
                    raise NotImplementedError("video inputs are not supported")
                path = item["path"]
                if vision_lora is not None or path not in cache:
                    patches, (t, gh, gw) = preprocess(load_image(path), vt.cfg)
                    entry = (vt.encode([patches], [(t, gh, gw)], lora=vision_lora), (t, gh // m, gw // m))
                    if vision_lora is not None:
                        feats.append(entry[0])
                        grids.append(entry[1])
                        continue
                    cache[path] = entry
                feats.append(cache[path][0])
                grids.append(cache[path][1])
        return (torch.cat(feats, 0), grids) if feats else (None, [])

    def _image_hook(self, media_rows: list[list[dict]], train: bool = False):
        """embed_hook placing image features on the image placeholder tokens.

        With vision LoRA targets and ``train``, the features carry an autograd
        graph to the tower's LoRA leaves (kept in ``self._vision_pass`` until
        the backward has run, see ``_finish_vision_pass``)."""
        from graspo_b200.models.vision import ImageInputs, VisionLoRA, image_grid, image_size

        if getattr(self.model, "vision", None) is None and getattr(self.model, "vision_cfg", None) is not None:
            # a pipeline stage after the first: the grids only (placeholder
            # counts and multimodal positions), no tower and no features
            vc = self.model.vision_cfg
            m = vc.spatial_merge_size
            grids = []
            for media in media_rows:
                for item in media or []:
                    if item.get("type") != "image":
                        raise NotImplementedError("video inputs are not supported")
                    t, gh, gw = image_grid(*image_size(item["path"]), vc)
                    grids.append((t, gh // m, gw // m))
            return ImageInputs(None, self._vision_pad_id, grids) if grids else None
        vlora = None
        if self.model.lora.vision_modules():
            vlora = VisionLoRA(self.model.lora, training=train)
            if train:
                self._vision_pass = vlora
        feats, grids = self._image_features(media_rows, vision_lora=vlora)
        if feats is None:
            return None
        return ImageInputs(feats, self._vision_pad_id, grids)

    def _finish_vision_pass(self) -> None:
        """Add the vision-tower LoRA gradients of the pass that just ran backward
        (only on the first rank of the TP group: every rank ran the same tower)."""
        vlora = getattr(self, "_vision_pass", None)
        if vlora is not None:
            vlora.accumulate(enabled=self.ps.tp_rank == 0)
            self._vision_pass = None

    def _generate_multimodal(self, samples, *, rollout_group_size: int, max_new_tokens: int,
                             max_prompt_length: int | None = None, temperature: float = 1.0, top_p: float = 1.0,
                             chat_template_kwargs: dict | None = None, **_: Any) -> list[NativeGeneration]:
        from graspo_b200.models.vision import expand_image_placeholders, image_grid, image_size, merged_tokens

        vc = getattr(self.model, "vision_cfg", None)
        if vc is None:
            raise NotImplementedError("this checkpoint has no vision tower (config.json vision_config)")
        t0 = time.monotonic()
        max_len = int(max_prompt_length or self.config.data.max_prompt_length)
        texts = [self.format_messages(s.messages, chat_template_kwargs, tools=s.tools) for s in samples]
        enc = self.tokenizer(texts, padding=False, add_special_tokens=False)
        pad = self._vision_pad_id
        prompts, media_rows = [], []
        for s, ids in zip(samples, enc["input_ids"], strict=True):
            media = [m for m in (s.media or []) if m.get("type") == "image"]
            counts = [merged_tokens(image_grid(*image_size(m["path"]), vc), vc) for m in media]
            ids = expand_image_placeholders(list(ids), pad, counts)
            if len(ids) > max_len:
                # keep the image tokens: drop text from the front of the prompt
                ids = ids[len(ids) - max_len:]
                if ids.count(pad) != sum(counts):
                    raise ValueError("max_prompt_length cuts into the image tokens of a prompt")
            prompts.append(ids)
            media_rows.append(media)
        tok = self.tokenizer
        eos = int(tok.eos_token_id)
        pad_tok = int(tok.pad_token_id if tok.pad_token_id is not None else eos)
        seed = int(self.config.training.seed) * 1_000_003 + self._train_batch_call_index
        seed += 7919 * (self.ps.dp_rank if self.ps else 0)
        res = self._engine.generate(prompts, group_size=rollout_group_size, max_new_tokens=max_new_tokens,
                                    temperature=temperature, top_p=top_p, eos_id=eos, pad_id=pad_tok,
                                    ignore_eos=bool(self.config.graspoflow.benchmark_ignore_eos), seed=seed,
                                    embed_hook=self._image_hook(media_rows))
        gens = self._generations(res, 0.0, time.monotonic() - t0)
        G = res.group_size
        for g, media in zip(gens, media_rows, strict=True):
            g.metadata["_media_rows"] = [media] * G
        return gens

    def generate_group(self, *, messages, tools=None, **kwargs) -> NativeGeneration:
        return self.generate_groups(message_batches=[messages], tool_batches=[tools], **kwargs)[0]

    def _generations(self, res, tokenize_sec: float, elapsed: float) -> list[NativeGeneration]:
        tok = self.tokenizer
        pad = int(tok.pad_token_id if tok.pad_token_id is not None else tok.eos_token_id)
        n, P = res.prompt_ids.shape
        G = res.group_size
        max_new = res.tokens.shape[1]
        seqs = torch.cat([res.prompt_ids.repeat_interleave(G, 0), res.tokens], dim=1)
        attn = seqs.ne(pad)
        action = torch.zeros((seqs.shape[0], seqs.shape[1] - 1), dtype=torch.bool)
        action[:, P - 1:] = True
        action &= attn[:, 1:]
        texts = tok.batch_decode(
            [row[:length].tolist() for row, length in zip(res.tokens, res.gen_lens, strict=True)],
            skip_special_tokens=True,
        )
        decode_tokens = int(sum(res.gen_lens))
        out = []
        for i in range(n):
            sl = slice(i * G, (i + 1) * G)
            out.append(NativeGeneration(
                sequences=seqs[sl], attention_mask=attn[sl], action_mask=action[sl], completions=texts[sl],
                prompt_len=P,
                metadata={
                    "adapter": "graspoflow", "rollout_group_size": G, "prefill_len": P,
                    "prompt_lens": [res.prompt_lens[i]], "generated_tokens_max": max_new,
                    "rollout_use_kv_cache": True, "rollout_paged_kv": self.fused,
                    "rollout_generation_split_count": int(getattr(res, "splits", 1)),
                    "rollout_generation_micro_batch_size": int(self.config.graspoflow.rollout_engine_batch) or n * G,
                    "rollout_empty_cache_after_split": bool(self.config.graspoflow.empty_cache_after_rollout_split),
                    "tokenize_sec": round(tokenize_sec / n, 6), "prefill_sec": round(res.prefill_sec / n, 6),
                    "decode_sec": round(res.decode_sec / n, 6), "decode_tokens": decode_tokens // n,
                    "decode_steps": res.decode_steps, "rollout_elapsed_sec": round(elapsed, 6),
                    "tp_rank": self.tp_rank, "tp_size": self.ps.tp_size,
                },
            ))
        return out

    def parse_completion(self, completion: str, sample: Any | None = None) -> ParsedCompletion:
        return parse_qwen_tool_completion(
            completion, expect_tool_calls=bool(getattr(sample, "expects_tool_calls", False)),
            tools=getattr(sample, "tools", None),
        )

    # ------------------------------------------------------------ log-probs
    def _token_budget_chunks(self, B: int, S: int, budget: int = 65536) -> list[slice]:
        per = max(1, budget // max(S, 1))
        return [slice(i, min(B, i + per)) for i in range(0, B, per)]

    @torch.no_grad()
    def sequence_log_probs(self, sequences, attention_mask, metadata: Any | None = None) -> torch.Tensor:
        dev = self.device
        seq = sequences.to(dev)
        mask = attention_mask.to(dev).bool()
        media_rows = (metadata or {}).get("_media_rows") if isinstance(metadata, dict) else None
        hook = self._image_hook(media_rows) if media_rows and any(media_rows) else None
        if self.ps.pp_size > 1:
            from graspo_b200.engine.pipeline import pp_logprobs, pp_logprobs_autograd

            if not self.fused:
                return pp_logprobs_autograd(self.model, self._comm, seq, mask, seq[:, 1:],
                                            chunk_rows=self._pp_chunk_rows(seq), embed_hook=hook)
            return pp_logprobs(self._fused, self._comm, seq, mask, seq[:, 1:], chunk_rows=self._pp_chunk_rows(seq),
                               embed_hook=hook)
        if hook is not None:
            return self._logprobs(seq, mask, train=False, embed_hook=hook)[0]
        outs = []
        for sl in self._token_budget_chunks(seq.shape[0], seq.shape[1]):
            outs.append(self._logprobs(seq[sl], mask[sl], train=False)[0])
        out = torch.cat(outs, 0)
        self._check_kernels()
        return out

    def _check_kernels(self) -> None:
        """Raise ``KernelTimeout`` if a bounded device wait gave up since the last check.

        A wait that ran out leaves the fused collective sites' arrival counters
        out of step with the host's expectations, so the sites are retired
        first (the next use builds fresh, zeroed buffers)."""
        if self.device.type != "cuda" or not self.fused:
            return
        from graspo_b200.ops._ext import KernelTimeout, check_errors

        try:
            check_errors(self.device)
        except KernelTimeout:
            red = getattr(self._fused, "_tp_red", None)
            if red is not None:
                red.close()
                self._fused._tp_red = None
            raise

    def _logprobs(self, seq, mask, *, train: bool, seed: int = 0, targets=None, embed_hook=None):
        """log p(targets) per position, [B, S-1] fp32 (targets default to seq[:, 1:]).

        In training the second return value carries what the backward needs.
        """
        B, S = seq.shape
        tgt = seq[:, 1:] if targets is None else targets
        if self.fused:
            from graspo_b200.models.fused import AttnMeta

            f = self._fused
            S_in = S
            if f.sp and (B * S) % self.ps.tp_size:
                # sequence parallelism splits the B*S tokens evenly over the TP ranks:
                # pad the sequence dimension with masked pad tokens
                while (B * S) % self.ps.tp_size:
                    S += 1
                pad = S - S_in
                seq = torch.cat([seq, seq.new_zeros(B, pad)], 1)
                mask = torch.cat([mask, mask.new_zeros(B, pad)], 1)
                tgt = torch.cat([tgt, tgt.new_zeros(B, pad)], 1)
            meta = AttnMeta.from_mask(mask)
            x0 = f.embed(seq)
            x0_graph = None
            if embed_hook is not None:
                x0 = embed_hook(seq, x0)
                if x0.requires_grad:
                    # image features with vision LoRA: the kernels see a plain tensor, the
                    # graph to the tower's LoRA leaves is kept for the backward
                    x0_graph, x0 = x0, x0.detach()
            xL, inputs = f.stage_forward(f.sp_shard(x0), meta, train=train, seed=seed, keep_inputs=train)
            hn, rstd = f.final_norm(xL)
            hn_all = f.sp_gather(hn)
            full = torch.zeros_like(seq)
            full[:, :-1] = tgt
            full = full.reshape(-1)
            logp_full, lse = f.token_logprobs(hn_all, full)
            logp = logp_full.view(B, S)[:, : S_in - 1].contiguous()
            return logp, ((meta, inputs, xL, hn_all, rstd, full, lse, x0_graph) if train else None)
        lora = EagerLoRA(self.model.lora, requires_grad=train)
        with torch.set_grad_enabled(train):
            if hasattr(self.model, "sequence_logprobs"):
                logp = self.model.sequence_logprobs(seq, mask, lora=lora, training=train, targets=tgt,
                                                    embed_hook=embed_hook)
            else:
                hidden = eager_stage_forward(self.model, seq, mask, lora=lora, training=train, embed_hook=embed_hook)
                logp = eager_token_logprobs(self.model, hidden[:, :-1], tgt)
        return logp, lora

    def _fused_backward_from_logp_grad(self, ctx, dlogp: torch.Tensor, seed: int) -> None:
        """Backprop d(loss)/d(logp) [B, S-1] through the head and all layers."""
        from graspo_b200.ops._ext import ext

        meta, inputs, xL, hn, rstd, full_targets, lse, x0_graph = ctx
        B, S = meta.B, meta.S
        g = torch.zeros(B, S, device=dlogp.device, dtype=torch.float32)
        g[:, : dlogp.shape[1]] = dlogp
        dhn = self._fused.token_logprobs_backward(hn, full_targets, lse, g.view(-1))
        dxL = torch.empty_like(xL)
        ext().rmsnorm_bwd(dhn, xL, self.model.norm, rstd, None, dxL, self.model.cfg.rms_norm_eps)
        del dhn
        dx0 = self._fused.stage_backward(inputs, dxL, meta, train=True, seed=seed,
                                         on_layer_done=self._dp_layer_hook())
        if x0_graph is not None:
            # into the vision tower through the image-feature rows of the embeddings
            torch.autograd.backward(x0_graph, self._fused.sp_gather(dx0).view_as(x0_graph))

    # ------------------------------------------------------------ training
    def check_replicas(self) -> None:
        """Debug check (``GRASPO_CHECK_REPLICAS=1``, after every optimize call):
        the LoRA parameters are bit-identical across data-parallel replicas and
        their TP-replicated part is identical across the tensor-parallel group."""
        from graspo_b200.parallel.state import replica_mismatches

        ps, lora = self.ps, self.model.lora
        bad = replica_mismatches(lora.params, ps.dp_group if ps.dp_size > 1 else None, name="lora (dp)")
        rep = lora.replicated_numel
        if rep:
            bad += replica_mismatches(lora.params[:rep], ps.tp_group if ps.tp_size > 1 else None, name="lora (tp)")
        if bad:
            raise RuntimeError("replicated LoRA state diverged: " + "; ".join(bad))

    def _dp_reducer(self):
        """The overlapped peer-memory DP gradient all-reduce (CUDA, DP > 1, fused
        path without pipeline stages); None where a library all-reduce is used."""
        ps = self.ps
        if not (ps.dp_size > 1 and ps.distributed and self.device.type == "cuda" and self.fused
                and ps.pp_size == 1):
            return None
        red = getattr(self, "_dp_red", None)
        if red is None:
            from graspo_b200.parallel.symm import DPGradReduce

            red = self._dp_red = DPGradReduce(self.model.lora.numel, ps.dp_group, self.device)
        return red

    def _dp_layer_hook(self):
        red = self._dp_reducer()
        if red is None:
            return None
        lora = self.model.lora
        return lambda layer: red.push(lora.grads, lora.layer_ranges(layer))

    def _dp_average_grads(self) -> None:
        ps = self.ps
        g = self.model.lora.grads
        red = self._dp_reducer()
        if red is not None:
            red.finish(g)
        elif ps.dp_size > 1 and ps.distributed:
            dist.all_reduce(g, group=ps.dp_group)
            g.div_(ps.dp_size)

    def _tp_sync_replicated_grads(self) -> None:
        ps = self.ps
        rep = self.model.lora.replicated_numel
        if ps.tp_size > 1 and ps.distributed and rep:
            dist.all_reduce(self.model.lora.grads[:rep], group=ps.tp_group)
        if ps.tp_size > 1 and ps.distributed and hasattr(self.model, "sync_partial_grads"):
            self.model.sync_partial_grads()

    def _pp_chunk_rows(self, seq) -> int:
        """Rows per pipeline micro-batch (graspoflow.pp_micro_batch_size, bounded by a token budget)."""
        rows = max(1, int(self.config.graspoflow.pp_micro_batch_size))
        return max(1, min(rows, 65536 // max(1, seq.shape[1])))

    def _backward_grpo(self, seq, mask, old, adv, act, clip_eps: float, seed: int, embed_hook=None):
        """Forward + GRPO loss + backward into the flat grad buffer; returns loss (device)."""
        B, S = seq.shape
        if self.ps.pp_size > 1 and not self.fused:
            from graspo_b200.engine.pipeline import pp_train_autograd

            self.loss_fn.policy_ratio_clip_eps = clip_eps

            def chunk_loss(logp_c, sl):
                return self.loss_fn(logp_c, old[sl], adv[sl], act[sl]) * ((sl.stop - sl.start) / B)

            loss = pp_train_autograd(self.model, self._comm, seq, mask, seq[:, 1:], chunk_loss,
                                     chunk_rows=self._pp_chunk_rows(seq), schedule=self.config.graspoflow.pp_schedule,
                                     max_inflight=int(self.config.graspoflow.pp_max_inflight_microbatches),
                                     clock=self._clock, embed_hook=embed_hook)
            self._finish_vision_pass()
            return loss
        if self.ps.pp_size > 1:
            from graspo_b200.engine.pipeline import pp_train
            from graspo_b200.ops._ext import ext

            old_c, adv_c, act_c = old.contiguous(), adv.contiguous(), act.to(torch.uint8).contiguous()

            def loss_fn(logp_c, sl):
                rows = sl.stop - sl.start
                loss = torch.zeros(1, device=seq.device, dtype=torch.float32)
                dlogp = torch.empty_like(logp_c)
                ext().grpo_loss(logp_c.contiguous(), old_c[sl], adv_c[sl], act_c[sl], clip_eps, rows / B, loss,
                                dlogp, None)
                return loss * (rows / B), dlogp

            loss = pp_train(self._fused, self._comm, seq, mask, seq[:, 1:], loss_fn, seed=seed,
                            chunk_rows=self._pp_chunk_rows(seq), schedule=self.config.graspoflow.pp_schedule,
                            max_inflight=int(self.config.graspoflow.pp_max_inflight_microbatches),
                            clock=self._clock, embed_hook=embed_hook)
            self._finish_vision_pass()
            return loss
        clock = self._clock
        if self.fused:
            from graspo_b200.ops._ext import ext

            with clock.time("micro_batch_forward_sec"):
                logp, ctx = self._logprobs(seq, mask, train=True, seed=seed, embed_hook=embed_hook)
            with clock.time("backward_sec"):
                loss = torch.zeros(1, device=seq.device, dtype=torch.float32)
                dlogp = torch.empty_like(logp)
                ext().grpo_loss(logp, old.contiguous(), adv.contiguous(), act.to(torch.uint8).contiguous(), clip_eps,
                                1.0, loss, dlogp, None)
                self._fused_backward_from_logp_grad(ctx, dlogp, seed)
                self._finish_vision_pass()
            return loss
        with clock.time("micro_batch_forward_sec"):
            logp, lora = self._logprobs(seq, mask, train=True, embed_hook=embed_hook)
            self.loss_fn.policy_ratio_clip_eps = clip_eps
            loss = self.loss_fn(logp, old, adv, act)
        with clock.time("backward_sec"):
            if torch.isfinite(loss):
                loss.backward()
                lora.accumulate_grads()
            self._finish_vision_pass()
        return loss.detach().reshape(1)

    def _shared_training_indices(self, count: int, optimize_round: int) -> list[int]:
        seed = int(self.config.training.seed) + self._train_batch_call_index * 1_000_003 + int(optimize_round)
        idx = list(range(count))
        random.Random(seed).shuffle(idx)
        return idx

    def train_batch(self, experiences: list[Experience], *, policy_ratio_clip_eps: float,
                    optimize_iterations_per_step: int, max_grad_norm: float) -> dict[str, Any]:
        tok = self.tokenizer
        pad = int(tok.pad_token_id if tok.pad_token_id is not None else tok.eos_token_id)
        bs = int(self.config.training.optimize_prompt_batch_size)
        if self.config.graspoflow.empty_cache_before_train and self.device.type == "cuda":
            torch.cuda.empty_cache()
        t0 = time.monotonic()
        from graspo_b200.utils.timing import PhaseClock

        self._clock = clock = PhaseClock(sync=self.config.graspoflow.synchronize_cuda_timing)
        lora_before = self.model.lora.parameter_norm()
        losses, norms = [], []
        round_secs = []
        steps = 0
        for rnd in range(int(optimize_iterations_per_step)):
            t_round = clock.now() if clock.sync else time.monotonic()
            idx = self._shared_training_indices(len(experiences), rnd)
            for start in range(0, len(idx) - bs + 1, bs):
                batch = [experiences[i] for i in idx[start : start + bs]]
                seq, att, old, adv, act = collate(batch, self.device, pad)
                self.optimizer.zero_grad()
                seed = (int(self.config.training.seed) << 20) ^ (self._train_batch_call_index << 10) ^ steps
                media_rows = [((e.metadata or {}).get("_media") or []) for e in batch]
                hook = self._image_hook(media_rows, train=True) if any(media_rows) else None
                loss = self._backward_grpo(seq, att, old, adv, act, policy_ratio_clip_eps, seed, embed_hook=hook)
                with clock.time("grad_sync_sec"):
                    # both are sums (they commute); the DP slices were already sent
                    # layer by layer during the backward
                    self._dp_average_grads()
                    self._tp_sync_replicated_grads()
                with clock.time("optimizer_step_sec"):
                    norm = self.optimizer.step(max_grad_norm, loss)
                losses.append(loss)
                norms.append(norm)
                steps += 1
            round_secs.append(round((clock.now() if clock.sync else time.monotonic()) - t_round, 6))
        self._train_batch_call_index += 1
        if os.environ.get("GRASPO_CHECK_REPLICAS", "0") == "1":
            self.check_replicas()
        loss_vals = [float(x) for x in torch.cat(losses).cpu()] if losses else []
        self._check_kernels()
        norm_vals = [float(x) for x in torch.cat([n.reshape(1) for n in norms]).cpu()] if norms else []
        skipped = int(self.optimizer.skipped.item())
        finite = [v for v in loss_vals if math.isfinite(v)]
        lora_after = self.model.lora.parameter_norm()
        metrics = {
            "optimized": steps > 0,
            "replay_buffer_trainable_completion_count": len(experiences),
            "optimizer_steps": steps,
            "skipped_nonfinite": skipped,
            "loss_mean": sum(finite) / len(finite) if finite else None,
            "grad_norm_mean": sum(norm_vals) / len(norm_vals) if norm_vals else None,
            "nonzero_grad_count": int((self.model.lora.grads != 0).any().item()) * len(self.model.lora.modules),
            "lora_norm_before": lora_before,
            "lora_norm_after": lora_after,
            "lora_norm_delta": lora_after - lora_before,
            "train_batch_total_sec": time.monotonic() - t0,
            "micro_batch_count": steps,
            "current_lr": self.optimizer.lr,
            "activation_checkpointing_enabled": bool(self.model.gradient_checkpointing),
            "optimize_round_sec": round_secs,
            **clock.summary(),
        }
        if clock.calls.get("pipeline_forward_calls"):
            metrics["pipeline_forward_calls"] = int(clock.calls["pipeline_forward_calls"])
        if self.ps.pp_size > 1:
            flow = self.config.graspoflow
            metrics.update({
                "pp_size": self.ps.pp_size, "pipeline_stage_rank": self.ps.pp_rank, "pp_schedule": flow.pp_schedule,
                "placement_strategy": flow.placement_strategy,
                "pipeline_pp_micro_batch_size": int(flow.pp_micro_batch_size),
                "pp_max_inflight_microbatches": int(flow.pp_max_inflight_microbatches),
                **clock.peaks,  # micro-batches per step and the most held at once on this stage
            })
        self._rank_event("train_batch_after", {"metrics": metrics})
        return self._aggregate_rank_metrics(metrics)

    def train_batch_sft(self, sft_batches: list[dict[str, Any]], *, optimize_iterations_per_step: int,
                        max_grad_norm: float) -> dict[str, Any]:
        """Supervised steps on tokenized batches (labels -100 on the prompt)."""
        tok = self.tokenizer
        pad = int(tok.pad_token_id if tok.pad_token_id is not None else tok.eos_token_id)
        fbs = int(self.config.graspoflow.forward_batch_size)
        losses, steps = [], 0
        t0 = time.monotonic()
        from graspo_b200.utils.timing import PhaseClock

        self._clock = clock = PhaseClock(sync=self.config.graspoflow.synchronize_cuda_timing)
        for _ in range(int(optimize_iterations_per_step)):
            for start in range(0, len(sft_batches), fbs):
                chunk = [self._sft_images(b) for b in sft_batches[start : start + fbs]]
                S = max(int(b_ids.shape[0]) for b_ids, _, _ in chunk)
                ids = torch.full((len(chunk), S), pad, dtype=torch.long)
                labels = torch.full((len(chunk), S), -100, dtype=torch.long)
                mask = torch.zeros((len(chunk), S), dtype=torch.bool)
                for i, (b_ids, b_labels, _) in enumerate(chunk):
                    n = int(b_ids.shape[0])
                    ids[i, :n], labels[i, :n], mask[i, :n] = b_ids, b_labels, True
                ids, labels, mask = ids.to(self.device), labels.to(self.device), mask.to(self.device)
                media_rows = [media for _, _, media in chunk]
                hook = self._image_hook(media_rows, train=True) if any(media_rows) else None
                self.optimizer.zero_grad()
                loss = self._backward_sft(ids, mask, labels, steps, embed_hook=hook)
                with clock.time("grad_sync_sec"):
                    self._tp_sync_replicated_grads()
                    self._dp_average_grads()
                with clock.time("optimizer_step_sec"):
                    self.optimizer.step(max_grad_norm, loss)
                losses.append(loss)
                steps += 1
        vals = [float(x) for x in torch.cat(losses).cpu()] if losses else []
        return self._aggregate_rank_metrics({
            "optimized": steps > 0, "optimizer_steps": steps,
            "loss_mean": sum(vals) / len(vals) if vals else None,
            "train_batch_total_sec": time.monotonic() - t0, "current_lr": self.optimizer.lr,
            **clock.summary(),
        })

    def _backward_sft(self, ids, mask, labels, step: int, embed_hook=None):
        """Token cross-entropy = -mean log p(label) over labelled positions
        (the quantity of core.loss.sft_cross_entropy_loss, without logits).
        ``embed_hook`` places the batch's image features (multimodal SFT,
        reference: models/qwen35_36/training.py:75-90)."""
        loss = self._backward_sft_pass(ids, mask, labels, step, embed_hook)
        self._finish_vision_pass()
        return loss

    def _backward_sft_pass(self, ids, mask, labels, step: int, embed_hook):
        tgt = labels[:, 1:]
        valid = tgt.ne(-100)
        denom = valid.sum().clamp_min(1)
        safe = torch.where(valid, tgt, torch.zeros_like(tgt))
        if self.ps.pp_size > 1 and not self.fused:
            from graspo_b200.engine.pipeline import pp_train_autograd

            def chunk_loss(logp_c, sl):
                return -(logp_c * valid[sl]).sum() / denom

            return pp_train_autograd(self.model, self._comm, ids, mask, safe, chunk_loss,
                                     chunk_rows=self._pp_chunk_rows(ids), schedule=self.config.graspoflow.pp_schedule,
                                     max_inflight=int(self.config.graspoflow.pp_max_inflight_microbatches),
                                     clock=self._clock, embed_hook=embed_hook)
        if self.ps.pp_size > 1:
            from graspo_b200.engine.pipeline import pp_train

            def loss_fn(logp_c, sl):
                v = valid[sl].float()
                return -(logp_c * v).sum().reshape(1) / denom, -(v / denom)

            return pp_train(self._fused, self._comm, ids, mask, safe, loss_fn, seed=step,
                            chunk_rows=self._pp_chunk_rows(ids), schedule=self.config.graspoflow.pp_schedule,
                            max_inflight=int(self.config.graspoflow.pp_max_inflight_microbatches),
                            clock=self._clock, embed_hook=embed_hook)
        clock = self._clock
        if self.fused:
            with clock.time("micro_batch_forward_sec"):
                logp, ctx = self._logprobs(ids, mask, train=True, seed=step, targets=safe, embed_hook=embed_hook)
                loss = -(logp * valid).sum() / denom
            with clock.time("backward_sec"):
                self._fused_backward_from_logp_grad(ctx, -(valid.float() / denom), step)
            return loss.detach().reshape(1)
        with clock.time("micro_batch_forward_sec"):
            logp, lora = self._logprobs(ids, mask, train=True, targets=safe, embed_hook=embed_hook)
            loss = -(logp * valid).sum() / denom
        with clock.time("backward_sec"):
            loss.backward()
            lora.accumulate_grads()
        return loss.detach().reshape(1)

    def _rank_event(self, phase: str, extra: dict[str, Any] | None = None) -> None:
        """Per-rank memory snapshot (and metrics) to logs/rank_metrics.rank_NNNNN.jsonl
        (reference: transformer_adapter.py:704-721)."""
        from graspo_b200.train.logger import append_rank_metrics, memory_snapshot

        ps = self.ps
        payload = {"event": "rank_memory", "phase": phase, "rank": self.rank,
                   "tp_rank": ps.tp_rank if ps else 0, "pp_rank": ps.pp_rank if ps else 0,
                   "dp_rank": ps.dp_rank if ps else 0, "device": str(self.device),
                   "memory": memory_snapshot(self.device)}
        if extra:
            payload.update(extra)
        try:
            append_rank_metrics(self.config.training.output_dir, self.rank, payload)
        except OSError:
            pass  # metrics are best effort; training goes on

    def _aggregate_rank_metrics(self, metrics: dict[str, Any]) -> dict[str, Any]:
        local = {"rank": self.rank, "tp_rank": self.tp_rank, **metrics}
        if not self.ps.distributed:
            return {**metrics, "rank": self.rank, "tp_rank": self.tp_rank, "rank_metrics": [local]}
        gathered: list[Any] = [None] * self.ps.world_size
        dist.all_gather_object(gathered, local)
        ranks = [g for g in gathered if g is not None]

        def mean(key):
            vals = [float(r[key]) for r in ranks if r.get(key) is not None]
            return sum(vals) / len(vals) if vals else None

        return {**metrics, "rank": self.rank, "tp_rank": self.tp_rank, "rank_metrics": ranks,
                "global_optimizer_steps_sum": sum(int(r.get("optimizer_steps") or 0) for r in ranks),
                "global_loss_mean": mean("loss_mean"), "global_grad_norm_mean": mean("grad_norm_mean"),
                "global_lora_norm_delta_mean": mean("lora_norm_delta")}

    # ------------------------------------------------------------ checkpoints
    def save_checkpoint(self, path: str | Path, *, trainer_state: dict[str, Any] | None = None) -> None:
        from graspo_b200.train.checkpoint import AsyncCheckpointWriter, save_rank_checkpoint

        path = Path(path)
        writer = self.__dict__.setdefault("_ckpt_writer", AsyncCheckpointWriter())
        if self.config.graspoflow.async_checkpoint and path.name != "final":
            writer.submit(self, path, trainer_state=trainer_state)
            return
        writer.wait(self)
        save_rank_checkpoint(self, path, trainer_state=trainer_state)

    def flush_checkpoints(self) -> None:
        """Finish a background checkpoint write, if one is in flight (all ranks call it)."""
        writer = self.__dict__.get("_ckpt_writer")
        if writer is not None:
            writer.wait(self)

    def abandon_checkpoints(self) -> None:
        """Stop waiting for an in-flight background checkpoint without completing it."""
        writer = self.__dict__.get("_ckpt_writer")
        if writer is not None:
            writer.abandon()

    def load_checkpoint(self, path: str | Path) -> dict[str, Any] | None:
        from graspo_b200.train.checkpoint import load_rank_checkpoint

        self.flush_checkpoints()
        return load_rank_checkpoint(self, Path(path))

    def close(self) -> None:
        self.flush_checkpoints()
        self._engine = None
        pstate.destroy()


class Qwen35Adapter(Qwen3Adapter):
    """Adapter of the Qwen3.5 / 3.6 hybrid family (gated DeltaNet + gated
    attention; reference: backends/graspoflow/models/qwen35_36/adapter.py:35-117).

    Training and log-probs run the model's autograd path (chunked delta rule,
    gradient checkpointing per layer), rollout runs ``HybridRolloutEngine``
    (per-row KV / conv / recurrent caches, the delta-rule decode step on the
    sm_100a kernel).  Heads are split over the tensor-parallel group (the
    model sums the row-parallel outputs, the adapter sums the replicated LoRA
    factors' gradients); text prompts only.
    """

    families = ("qwen3_5_text",)
    autograd_pipeline = True

    @property
    def model_class(self):
        from graspo_b200.models.qwen35 import Qwen35Model

        return Qwen35Model

    @property
    def fused(self) -> bool:
        return False

    def _eager_engine(self):
        from graspo_b200.models.qwen35 import HybridRolloutEngine

        return HybridRolloutEngine(self.model, comm=self._comm)
