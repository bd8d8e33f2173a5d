"""Model parity against the Hugging Face implementations (CPU, fp32).

The eager forward of both model families is compared with the
``transformers`` modules of the same architecture on the same random-init
checkpoint: ``Qwen3ForCausalLM`` for the dense family and
``Qwen3_5ForCausalLM`` (gated DeltaNet + gated attention, partial RoPE,
(1 + w) norms) for the hybrid one, ``Qwen3_5VisionModel`` for the vision
tower (patch embedding, resampled position table, 2-D rotary, merger) on
images of two grid sizes.  Left-padded rows get the positions that
the training and rollout paths use (count of real tokens before them).
Reference behaviour: models/qwen3/model.py:250-365 and
models/qwen35_36/model.py:486-543, both built to reproduce the HF modules.
"""

import json

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _batch(vocab: int):
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, vocab - 8, (2, 80), generator=g)
    mask = torch.ones(2, 80, dtype=torch.bool)
    mask[1, :13] = False
    pos = (mask.long().cumsum(-1) - 1).clamp_min(0)
    return ids, mask, pos


def _hf_logprobs(logits, ids):
    return torch.log_softmax(logits[:, :-1].float(), -1).gather(-1, ids[:, 1:, None]).squeeze(-1)


def test_qwen3_dense_matches_transformers(tmp_path):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model, eager_sequence_logprobs
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import TINY, write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "q3", TINY, seed=1, std=0.05, dtype=torch.float32, device="cpu",
                                  with_tokenizer=False)
    cfg = json.loads((path / "config.json").read_text())
    hc = Qwen3Config(**cfg)
    hc._attn_implementation = "eager"
    hf = Qwen3ForCausalLM(hc).float().eval()
    from safetensors.torch import load_file

    state = {}
    for f in sorted(path.glob("*.safetensors")):
        state.update(load_file(str(f)))
    missing, unexpected = hf.load_state_dict(state, strict=False)
    assert not [k for k in missing if "rotary" not in k] and not unexpected, (missing, unexpected)
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), dtype=torch.float32,
                   device=torch.device("cpu"))
    ids, mask, pos = _batch(cfg["vocab_size"])
    with torch.no_grad():
        ref = _hf_logprobs(hf(input_ids=ids, attention_mask=mask.long(), position_ids=pos).logits, ids)
        got = eager_sequence_logprobs(m, ids, mask)
    valid = mask[:, :-1] & mask[:, 1:]
    assert (got - ref).abs()[valid].max().item() < 1e-3


def test_qwen35_hybrid_matches_transformers(tmp_path):
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_TINY, write_qwen35_checkpoint

    path = write_qwen35_checkpoint(tmp_path / "q35", QWEN35_TINY, seed=1, std=0.05, dtype=torch.float32,
                                   with_tokenizer=False)
    text = json.loads((path / "config.json").read_text())["text_config"]
    hc = Qwen3_5TextConfig(**text)
    hc._attn_implementation = "eager"
    hf = Qwen3_5ForCausalLM(hc).float().eval()
    from safetensors.torch import load_file

    state = {k.replace("model.language_model.", "model."): v
             for k, v in load_file(str(path / "model.safetensors")).items()}
    missing, unexpected = hf.load_state_dict(state, strict=False)
    assert not [k for k in missing if "rotary" not in k] and not unexpected, (missing, unexpected)
    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), dtype=torch.float32)
    ids, mask, pos = _batch(QWEN35_TINY["vocab_size"])
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask.long(), position_ids=pos).logits
        got = m.logits(m.forward(ids, mask))
    assert (got - ref).abs()[mask].max().item() < 1e-3
    lp = m.sequence_logprobs(ids, mask)
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp - _hf_logprobs(ref, ids)).abs()[valid].max().item() < 1e-3


def test_vision_tower_matches_transformers(tmp_path):
    """The native ViT + 2x2 merger equals ``Qwen3_5VisionModel`` on the same weights and patches."""
    from safetensors.torch import load_file
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5VisionModel

    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.vision import VisionConfig, VisionTower, preprocess
    from graspo_b200.utils.synth import TINY, VIT_TINY, add_vision_tower, write_qwen3_checkpoint

    path = add_vision_tower(write_qwen3_checkpoint(tmp_path / "vl", TINY, seed=1, device="cpu", dtype=torch.float32,
                                                   with_tokenizer=False), VIT_TINY, seed=2, std=0.2,
                            dtype=torch.float32)
    vc = json.loads((path / "config.json").read_text())["vision_config"]
    hc = Qwen3_5VisionConfig(**vc)
    hc._attn_implementation = "eager"
    hf = Qwen3_5VisionModel(hc).float().eval()
    state = {k[len("model.visual."):]: v for k, v in load_file(str(path / "model-vision.safetensors")).items()}
    missing, unexpected = hf.load_state_dict(state, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    cfg = VisionConfig.from_dict(vc)
    vt = VisionTower(cfg, SafetensorIndex(path), "model.visual", dtype=torch.float32, device=torch.device("cpu"))
    g = torch.Generator().manual_seed(0)
    images = [torch.randint(0, 256, (96, 128, 3), dtype=torch.uint8, generator=g),
              torch.randint(0, 256, (64, 64, 3), dtype=torch.uint8, generator=g)]
    pre = [preprocess(img, cfg) for img in images]
    with torch.no_grad():
        mine = vt.encode([p for p, _ in pre], [grid for _, grid in pre])
        out = hf(torch.cat([p for p, _ in pre]), grid_thw=torch.tensor([list(grid) for _, grid in pre]))
    ref = out.pooler_output
    assert mine.shape == ref.shape
    assert (mine - ref).abs().max().item() < 1e-3 * ref.abs().max().item()
