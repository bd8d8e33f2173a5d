"""Vision tower: native ViT + 2x2 patch merger feeding image features to the decoder.

Architecture of the Qwen3.5 / Qwen3-VL vision encoder (the reference runs the
Hugging Face module; reference: backends/graspoflow/models/qwen3/model.py:170-232,
qwen35_36/model.py:263-286), written here as plain tensor code:

* patch embedding: each image is cut into 16 x 16 patches of 3 channels and 2
  (duplicated) frames; the 3-D convolution with kernel == stride is a single
  linear map of the flattened 1536-value patch (one GEMM);
* a learned position table on a 48 x 48 grid, bilinearly resampled to the
  image's patch grid;
* 2-D rotary embedding on the attention heads (row and column frequencies);
* ``depth`` pre-LayerNorm blocks: bidirectional multi-head attention inside
  each image (QKV / output projections with bias), GELU(tanh) MLP;
* merger: LayerNorm, every 2 x 2 block of neighbouring patches concatenated,
  Linear -> GELU -> Linear into the decoder's hidden size.

Patches are kept in merge-block order (rows of 2 x 2 blocks), so the merger's
concatenation is a reshape.  ``preprocess`` turns an RGB uint8 image into
that patch layout (CLIP mean / std normalisation, sides rounded to a multiple
of 32 pixels).  The decoder receives one feature per merged block in place of
each image placeholder token (``scatter_image_features``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

MEAN = (0.48145466, 0.4578275, 0.40821073)
STD = (0.26862954, 0.26130258, 0.27577711)


@dataclass
class VisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    spatial_merge_size: int = 2
    temporal_patch_size: int = 2
    out_hidden_size: int = 4096
    num_position_embeddings: int = 2304

    @staticmethod
    def from_dict(d: dict) -> "VisionConfig":
        keys = VisionConfig.__dataclass_fields__.keys()
        return VisionConfig(**{k: d[k] for k in keys if k in d})

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2


def _resized(H: int, W: int, cfg: VisionConfig) -> tuple[int, int]:
    """The image size ``preprocess`` resamples to: each side rounded to a whole
    number of merge blocks (at least one)."""
    unit = cfg.patch_size * cfg.spatial_merge_size
    return max(unit, round(H / unit) * unit), max(unit, round(W / unit) * unit)


def image_grid(height: int, width: int, cfg: VisionConfig) -> tuple[int, int, int]:
    """The patch grid ``(1, gh, gw)`` that ``preprocess`` gives an image of this size."""
    h2, w2 = _resized(int(height), int(width), cfg)
    return 1, h2 // cfg.patch_size, w2 // cfg.patch_size


def image_size(path: str) -> tuple[int, int]:
    """(height, width) of an image file, read from its header."""
    from PIL import Image

    with Image.open(path) as im:
        w, h = im.size
    return h, w


def preprocess(image: torch.Tensor, cfg: VisionConfig) -> tuple[torch.Tensor, tuple[int, int, int]]:
    """uint8 [H, W, 3] -> (patches [gh * gw, patch_dim] in merge-block order, (1, gh, gw))."""
    img = image.permute(2, 0, 1).float()[None] / 255.0                       # [1, 3, H, W]
    H, W = img.shape[-2:]
    h2, w2 = _resized(H, W, cfg)
    if (h2, w2) != (H, W):
        img = F.interpolate(img, size=(h2, w2), mode="bicubic", align_corners=False)
    mean = torch.tensor(MEAN).view(1, 3, 1, 1)
    std = torch.tensor(STD).view(1, 3, 1, 1)
    img = ((img - mean) / std)[0]                                             # [3, h2, w2]
    p, m, t = cfg.patch_size, cfg.spatial_merge_size, cfg.temporal_patch_size
    gh, gw = h2 // p, w2 // p
    frames = img[None].expand(t, -1, -1, -1)                                  # an image is t equal frames
    x = frames.reshape(t, 3, gh // m, m, p, gw // m, m, p)
    x = x.permute(2, 5, 3, 6, 1, 0, 4, 7)                                     # (bh, bw, mh, mw, C, t, p, p)
    return x.reshape(gh * gw, cfg.patch_dim).contiguous(), (1, gh, gw)


def load_image(path: str) -> torch.Tensor:
    from PIL import Image

    with Image.open(path) as im:
        return torch.from_numpy(__import__("numpy").asarray(im.convert("RGB"), dtype="uint8").copy())


_VISION_LINEARS = ("attn.qkv", "attn.proj", "mlp.linear_fc1", "mlp.linear_fc2")


def vision_lora_modules(cfg: VisionConfig, targets) -> list:
    """LoRA modules of the vision tower for the enabled targets (reference names
    ``visual.blocks.<i>.attn.qkv`` ... and ``visual.merger.linear_fc1/2``; presets
    ``vision_merger`` and ``vision_common``).  The tower is replicated over
    tensor parallelism, so both factors are unsharded."""
    from graspo_b200.core.lora_targets import lora_target_enabled
    from graspo_b200.models.lora import LoRAModule

    H, inter = cfg.hidden_size, cfg.intermediate_size
    merged = H * cfg.spatial_merge_size ** 2
    dims = {"attn.qkv": (H, 3 * H), "attn.proj": (H, H), "mlp.linear_fc1": (H, inter), "mlp.linear_fc2": (inter, H)}
    spec = [(f"blocks.{i}.{name}", *dims[name]) for i in range(cfg.depth) for name in _VISION_LINEARS]
    spec += [("merger.linear_fc1", merged, merged), ("merger.linear_fc2", merged, cfg.out_hidden_size)]
    out = []
    for path, d_in, d_out in spec:
        target = f"visual.{path}"
        if not lora_target_enabled(targets, target):
            continue
        out.append(LoRAModule(module_name=target, target_name=target, hf_module_path=f"model.visual.{path}",
                              layer=-1, kind="vision", shard_kind="none", in_full=d_in, out_full=d_out,
                              in_local=d_in, out_local=d_out))
    return out


class VisionLoRA:
    """Autograd leaves of the vision-tower LoRA factors for one training pass.

    The leaves share storage with the adapter's fp32 master weights; after the
    backward, ``accumulate`` adds their gradients into the flat gradient
    buffer.  Every tensor-parallel rank runs the same tower on the same images,
    so only one rank of the group adds them (the group's gradient sum of the
    replicated factors then yields the gradient once)."""

    def __init__(self, adapter, *, training: bool) -> None:
        self.adapter = adapter
        self.training = training
        self.modules = {m.module_name: m for m in adapter.vision_modules()}
        self.leaves = {name: (m.a.detach().requires_grad_(training), m.b.detach().requires_grad_(training))
                       for name, m in self.modules.items()}

    def delta(self, name: str, x: torch.Tensor) -> torch.Tensor | None:
        pair = self.leaves.get(name)
        if pair is None:
            return None
        a, b = pair
        p = self.adapter.dropout
        xin = F.dropout(x, p, True) if (self.training and p > 0) else x
        return F.linear(F.linear(xin.float(), a), b) * self.adapter.scaling

    def accumulate(self, enabled: bool = True) -> None:
        for name, m in self.modules.items():
            a, b = self.leaves[name]
            if enabled and a.grad is not None:
                m.a_grad.add_(a.grad)
            if enabled and b.grad is not None:
                m.b_grad.add_(b.grad)
            a.grad = b.grad = None


class VisionTower:
    """Vision encoder (weights under ``<prefix>.``), frozen; LoRA on its linears when enabled."""

    def __init__(self, cfg: VisionConfig, loader, prefix: str, *, dtype: torch.dtype, device: torch.device) -> None:
        self.cfg, self.dtype, self.device = cfg, dtype, device

        def load(name):
            return loader.get(f"{prefix}.{name}").to(device=device, dtype=dtype)

        self.patch_w = load("patch_embed.proj.weight").reshape(cfg.hidden_size, cfg.patch_dim)
        self.patch_b = load("patch_embed.proj.bias")
        self.pos_table = load("pos_embed.weight")
        self.blocks = []
        for i in range(cfg.depth):
            b = f"blocks.{i}"
            self.blocks.append({n: load(f"{b}.{n}") for n in (
                "norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias", "attn.qkv.weight", "attn.qkv.bias",
                "attn.proj.weight", "attn.proj.bias", "mlp.linear_fc1.weight", "mlp.linear_fc1.bias",
                "mlp.linear_fc2.weight", "mlp.linear_fc2.bias")})
        self.merger = {n: load(f"merger.{n}") for n in (
            "norm.weight", "norm.bias", "linear_fc1.weight", "linear_fc1.bias", "linear_fc2.weight", "linear_fc2.bias")}
        hd = cfg.hidden_size // cfg.num_heads
        self.head_dim = hd
        quarter = hd // 2
        self.rot_inv = (1.0 / (10000.0 ** (torch.arange(0, quarter, 2, dtype=torch.float32) / quarter))).to(device)

    def _pos_embed(self, gh: int, gw: int) -> torch.Tensor:
        n = int(math.isqrt(self.cfg.num_position_embeddings))
        table = self.pos_table.float().view(n, n, -1).permute(2, 0, 1)[None]   # [1, C, n, n]
        grid = F.interpolate(table, size=(gh, gw), mode="bilinear", align_corners=True)[0]  # [C, gh, gw]
        m = self.cfg.spatial_merge_size
        grid = grid.permute(1, 2, 0).reshape(gh // m, m, gw // m, m, -1).permute(0, 2, 1, 3, 4)
        return grid.reshape(gh * gw, -1)

    def _rotary(self, gh: int, gw: int) -> tuple[torch.Tensor, torch.Tensor]:
        m = self.cfg.spatial_merge_size
        rows = torch.arange(gh, device=self.device).view(gh // m, 1, m, 1).expand(gh // m, gw // m, m, m)
        cols = torch.arange(gw, device=self.device).view(1, gw // m, 1, m).expand(gh // m, gw // m, m, m)
        fr = rows.reshape(-1, 1).float() * self.rot_inv
        fc = cols.reshape(-1, 1).float() * self.rot_inv
        emb = torch.cat([fr, fc], -1)
        emb = torch.cat([emb, emb], -1)                                         # [N, head_dim]
        return emb.cos(), emb.sin()

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], -1)
        return x * cos[:, None] + rot * sin[:, None]

    def encode(self, patches: list[torch.Tensor], grids: list[tuple[int, int, int]],
               lora: VisionLoRA | None = None) -> torch.Tensor:
        """Per-image patches -> merged features [sum(gh * gw / 4), out_hidden], images in order.

        Without ``lora`` (or with LoRA leaves that need no gradient) this runs
        without an autograd graph."""
        if lora is None or not lora.training:
            with torch.no_grad():
                return self._encode(patches, grids, lora)
        return self._encode(patches, grids, lora)

    def _encode(self, patches, grids, lora):
        cfg = self.cfg
        outs = []

        def lin(x, w, bias, name):
            y = F.linear(x, w, bias)
            d = lora.delta(name, x) if lora is not None else None
            return y if d is None else y + d.to(y.dtype)
        for pt, (_, gh, gw) in zip(patches, grids, strict=True):
            x = F.linear(pt.to(self.device, self.dtype), self.patch_w, self.patch_b)
            x = (x.float() + self._pos_embed(gh, gw)).to(self.dtype)
            cos, sin = self._rotary(gh, gw)
            N = x.shape[0]
            for bi, blk in enumerate(self.blocks):
                pre = f"visual.blocks.{bi}."
                h = F.layer_norm(x, (cfg.hidden_size,), blk["norm1.weight"], blk["norm1.bias"], 1e-6)
                qkv = lin(h, blk["attn.qkv.weight"], blk["attn.qkv.bias"], pre + "attn.qkv").view(N, 3, cfg.num_heads, -1)
                q = self._rope(qkv[:, 0].float(), cos, sin).to(self.dtype)
                k = self._rope(qkv[:, 1].float(), cos, sin).to(self.dtype)
                v = qkv[:, 2]
                o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                   v.transpose(0, 1)[None])[0].transpose(0, 1).reshape(N, -1)
                x = x + lin(o, blk["attn.proj.weight"], blk["attn.proj.bias"], pre + "attn.proj")
                h = F.layer_norm(x, (cfg.hidden_size,), blk["norm2.weight"], blk["norm2.bias"], 1e-6)
                h = F.gelu(lin(h, blk["mlp.linear_fc1.weight"], blk["mlp.linear_fc1.bias"], pre + "mlp.linear_fc1"),
                           approximate="tanh")
                x = x + lin(h, blk["mlp.linear_fc2.weight"], blk["mlp.linear_fc2.bias"], pre + "mlp.linear_fc2")
            mg = self.merger
            h = F.layer_norm(x, (cfg.hidden_size,), mg["norm.weight"], mg["norm.bias"], 1e-6)
            h = h.reshape(-1, cfg.hidden_size * cfg.spatial_merge_size ** 2)
            h = F.gelu(lin(h, mg["linear_fc1.weight"], mg["linear_fc1.bias"], "visual.merger.linear_fc1"))
            outs.append(lin(h, mg["linear_fc2.weight"], mg["linear_fc2.bias"], "visual.merger.linear_fc2"))
        return torch.cat(outs, 0)


def merged_tokens(grid: tuple[int, int, int], cfg: VisionConfig) -> int:
    t, gh, gw = grid
    return t * (gh // cfg.spatial_merge_size) * (gw // cfg.spatial_merge_size)


def expand_image_placeholders(ids: list[int], pad_id: int, counts: list[int]) -> list[int]:
    """Replace the k-th image placeholder token with counts[k] copies of it."""
    out, k = [], 0
    for t in ids:
        if t == pad_id and k < len(counts):
            out.extend([pad_id] * counts[k])
            k += 1
        else:
            out.append(t)
    if k != len(counts):
        raise ValueError(f"prompt has {k} image placeholders for {len(counts)} images")
    return out


def scatter_image_features(x: torch.Tensor, ids: torch.Tensor, pad_id: int, feats: torch.Tensor) -> torch.Tensor:
    """x [T, H] token embeddings of ids [T]: placeholder rows take the image features in order."""
    sel = ids.reshape(-1) == pad_id
    n = int(sel.sum())
    if n != feats.shape[0]:
        raise ValueError(f"{n} image placeholder tokens for {feats.shape[0]} image features")
    x[sel] = feats.to(x.dtype)
    return x


class ImageInputs:
    """``embed_hook`` of a batch with images: places the features of every
    image (rows in order, images in order) on the placeholder embeddings, and
    carries each image's merged grid ``(t, h, w)`` so a decoder with
    multimodal RoPE can give the placeholders their 3-D positions."""

    def __init__(self, feats: torch.Tensor | None, pad_id: int, grids: list[tuple[int, int, int]]) -> None:
        # feats is None on pipeline stages after the first: they only need the
        # grids (multimodal positions), the features enter with the embeddings
        self.feats, self.pad_id, self.grids = feats, int(pad_id), list(grids)
        self._cut: list[tuple[torch.Tensor, torch.Tensor]] = []

    def rows(self, ids: torch.Tensor, sl: slice) -> "ImageInputs":
        """The images of rows ``sl`` of the batch ``ids`` [B, S]: each row's
        placeholders take the next images' features, in row order."""
        per_row = (ids == self.pad_id).sum(1).tolist()
        f0 = sum(per_row[: sl.start])
        f1 = f0 + sum(per_row[sl])
        bounds, acc = [0], 0
        for t, h, w in self.grids:
            acc += t * h * w
            bounds.append(acc)
        if f0 not in bounds or f1 not in bounds:
            raise ValueError("image placeholder counts do not match the image grids")
        feats = self.feats[f0:f1] if self.feats is not None else None
        return ImageInputs(feats, self.pad_id, self.grids[bounds.index(f0) : bounds.index(f1)])

    def split_rows(self, ids: torch.Tensor, chunks: list[slice]) -> list["ImageInputs"]:
        """One ``rows`` view per micro-batch.  Features that carry a graph to
        the vision tower (LoRA on the tower, training) are cut from it here:
        each micro-batch gets leaf features, and ``backward_into_tower`` sends
        their gradients through the tower in one pass after the last
        micro-batch's backward."""
        parts = []
        for sl in chunks:
            sub = self.rows(ids, sl)
            if sub.feats is not None and sub.feats.requires_grad:
                leaf = sub.feats.detach().requires_grad_(True)
                self._cut.append((sub.feats, leaf))
                sub.feats = leaf
            parts.append(sub)
        return parts

    def backward_into_tower(self) -> None:
        pairs = [(g, leaf.grad) for g, leaf in self._cut if leaf.grad is not None]
        self._cut = []
        if pairs:
            torch.autograd.backward([g for g, _ in pairs], [d.to(g.dtype) for g, d in pairs])

    def __call__(self, ids: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 2:
            return scatter_image_features(x, ids, self.pad_id, self.feats)
        scatter_image_features(x.view(-1, x.shape[-1]), ids, self.pad_id, self.feats)
        return x
