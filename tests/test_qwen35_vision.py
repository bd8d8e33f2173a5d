"""Qwen3.5 with images (CPU, fp32).

* The hybrid decoder fed the native vision tower's features on the image
  placeholders, with interleaved multimodal RoPE positions, gives the logits
  of ``transformers``' ``Qwen3_5ForConditionalGeneration`` (pixel values,
  image grids, left padding).
* Cached greedy decoding after an image prompt continues from the prompt's
  largest position: re-scoring the whole prompt + completion in one pass
  picks the same tokens.
Reference behaviour: models/qwen35_36/model.py:248-330, 372-461 (image
features scattered into the embeddings, 3-D positions, decode deltas).
"""

import json

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _setup(tmp_path):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model
    from graspo_b200.models.vision import ImageInputs, merged_tokens, preprocess
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_TINY, VIT_TINY, add_vision_tower, write_qwen35_checkpoint

    dims = dict(QWEN35_TINY, head_dim=64)          # 16 rotary frequencies: all three position components used
    path = add_vision_tower(write_qwen35_checkpoint(tmp_path / "q35vl", dims, seed=1, std=0.05, dtype=torch.float32,
                                                    with_tokenizer=False), VIT_TINY, seed=2, std=0.2,
                            dtype=torch.float32)
    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), dtype=torch.float32)
    pad_id = json.loads((path / "config.json").read_text())["image_token_id"]
    g = torch.Generator().manual_seed(0)
    images = [torch.randint(0, 256, (96, 128, 3), dtype=torch.uint8, generator=g),
              torch.randint(0, 256, (64, 96, 3), dtype=torch.uint8, generator=g)]
    pre = [preprocess(img, m.vision.cfg) for img in images]
    n_tok = [merged_tokens(grid, m.vision.cfg) for _, grid in pre]
    # row 0: text, image 0, text; row 1 (left-padded): text, image 1, text
    rows = [[11, 12, 13] + [pad_id] * n_tok[0] + [14, 15, 16, 17],
            [21, 22] + [pad_id] * n_tok[1] + [23, 24]]
    S = max(len(r) for r in rows)
    ids = torch.full((2, S), 3, dtype=torch.long)
    mask = torch.zeros(2, S, dtype=torch.bool)
    for i, r in enumerate(rows):
        ids[i, S - len(r):] = torch.tensor(r)
        mask[i, S - len(r):] = True
    mrg = m.vision.cfg.spatial_merge_size
    with torch.no_grad():
        feats = m.vision.encode([p for p, _ in pre], [grid for _, grid in pre])
    hook = ImageInputs(feats, pad_id, [(t, h // mrg, w // mrg) for _, (t, h, w) in pre])
    return path, m, ids, mask, pre, hook, pad_id


def test_qwen35_image_prompt_matches_transformers(tmp_path):
    from safetensors.torch import load_file
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration

    path, m, ids, mask, pre, hook, pad_id = _setup(tmp_path)
    raw = json.loads((path / "config.json").read_text())
    hc = Qwen3_5Config(text_config=raw["text_config"], vision_config=raw["vision_config"], image_token_id=pad_id)
    hc._attn_implementation = "eager"
    hc.text_config._attn_implementation = "eager"
    hc.vision_config._attn_implementation = "eager"
    hf = Qwen3_5ForConditionalGeneration(hc).float().eval()
    state = {}
    for f in sorted(path.glob("*.safetensors")):
        state.update(load_file(str(f)))
    missing, unexpected = hf.load_state_dict(state, strict=False)
    assert not [k for k in missing if "rotary" not in k] and not unexpected, (missing, unexpected)
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask.long(), pixel_values=torch.cat([p for p, _ in pre]),
                 image_grid_thw=torch.tensor([list(grid) for _, grid in pre]),
                 mm_token_type_ids=(ids == pad_id).int()).logits
        got = m.logits(m.forward(ids, mask, embed_hook=hook))
    err = (got - ref).abs()[mask].max().item()
    assert err < 1e-3 * max(1.0, ref.abs().max().item()), err
    # text-only positions would differ: the image really moves the positions
    with torch.no_grad():
        flat = m.logits(m.forward(ids, mask, embed_hook=lambda i, x: hook(i, x)))
    assert (flat - ref).abs()[mask].max().item() > 10 * err


def test_qwen35_image_decoding_continues_the_positions(tmp_path):
    from graspo_b200.models.qwen35 import HybridRolloutEngine

    _, m, ids, mask, pre, hook, pad_id = _setup(tmp_path)
    prompts = [ids[i][mask[i]].tolist() for i in range(2)]
    res = HybridRolloutEngine(m).generate(prompts, group_size=1, max_new_tokens=5, temperature=0.0, top_p=1.0,
                                          eos_id=508, pad_id=3, ignore_eos=True, seed=0, embed_hook=hook)
    full = torch.cat([res.prompt_ids, res.tokens], 1)
    fmask = torch.cat([res.prompt_ids != 3, torch.ones_like(res.tokens, dtype=torch.bool)], 1)   # 3: prompt padding
    with torch.no_grad():
        logits = m.logits(m.forward(full, fmask, embed_hook=hook))
    P = res.prompt_ids.shape[1]
    greedy = logits[:, P - 1 : P - 1 + 5].argmax(-1)
    assert torch.equal(greedy, res.tokens), (greedy, res.tokens)


def _tp2_image_worker(rank, world, tmp, ref_file):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model
    from graspo_b200.models.vision import ImageInputs
    from graspo_b200.parallel import state as pstate

    ps = pstate.initialize(2, 1, 0, timeout_sec=120, device="cpu")
    ref = torch.load(ref_file)
    path = ref["path"]
    hook = ImageInputs(ref["feats"], int(ref["pad_id"]), [tuple(g) for g in ref["grids"].tolist()])
    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, dtype=torch.float32)
    assert m.vision is not None and m.nq_l * 2 == m.nq
    with torch.no_grad():
        got = m.logits(m.forward(ref["ids"], ref["mask"], embed_hook=hook))
    mask = ref["mask"]
    assert (got - ref["logits"]).abs()[mask].max().item() < 1e-4
    pstate.destroy()


def test_qwen35_image_prompt_tp2_matches_tp1(tmp_path):
    """Heads split over two CPU ranks, vision tower and multimodal positions
    replicated on each: the image-prompt logits of TP = 1."""
    import os

    from tests.dist_util import run_world

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    path, m, ids, mask, pre, hook, pad_id = _setup(tmp_path)
    with torch.no_grad():
        logits = m.logits(m.forward(ids, mask, embed_hook=hook))
    ref_file = tmp_path / "ref.pt"
    torch.save({"path": str(path), "ids": ids, "mask": mask, "feats": hook.feats, "pad_id": pad_id,
                "grids": torch.tensor(hook.grids), "logits": logits}, ref_file)
    run_world(2, _tp2_image_worker, str(tmp_path), str(ref_file), timeout=600)
