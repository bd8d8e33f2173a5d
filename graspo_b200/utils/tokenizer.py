"""Deterministic offline tokenizer that Hugging Face ``AutoTokenizer`` can load.

There is no network access for real Qwen tokenizer files, so benchmarks and
tests use a byte-level tokenizer written with the ``tokenizers`` library:

* ids 0..255: the 256 byte symbols (GPT-2 style byte-to-unicode alphabet), so
  any UTF-8 text round-trips;
* every other id up to ``vocab_size`` decodes to a visible placeholder
  ``<t12345>`` (a random-init model samples those ids, and completions must
  still decode to text);
* ``<|endoftext|>`` (EOS/pad), ``<|im_start|>``, ``<|im_end|>`` at the Qwen ids
  151643-151645 when the vocabulary is large enough, else at the top;
* a Qwen-style chat template (``<|im_start|>role\\ncontent<|im_end|>``) with
  tools rendered as JSON into the system turn.
"""

from __future__ import annotations

import json
from pathlib import Path

CHAT_TEMPLATE = (
    "{% if tools %}<|im_start|>system\n"
    "{% if messages[0]['role'] == 'system' %}{{ messages[0]['content'] }}\n\n{% endif %}"
    "# Tools\n{{ tools | tojson }}<|im_end|>\n"
    "{% endif %}"
    "{% for message in messages %}"
    "{% if not (tools and loop.first and message['role'] == 'system') %}"
    "<|im_start|>{{ message['role'] }}\n"
    "{% if message['content'] is string %}{{ message['content'] }}"
    "{% else %}{% for part in message['content'] %}"
    "{% if part['type'] == 'text' %}{{ part['text'] }}{% else %}<|vision_pad|>{% endif %}"
    "{% endfor %}{% endif %}<|im_end|>\n"
    "{% endif %}"
    "{% endfor %}"
    "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}"
)


def _bytes_to_unicode() -> dict[int, str]:
    # The reversible byte -> printable character map used by byte-level BPE
    # (printable Latin-1 bytes map to themselves, the rest to 256+n).
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    chars = list(keep)
    n = 0
    for b in range(256):
        if b not in keep:
            keep.append(b)
            chars.append(256 + n)
            n += 1
    return dict(zip(keep, (chr(c) for c in chars), strict=True))


def special_token_ids(vocab_size: int) -> dict[str, int]:
    base = 151643 if vocab_size >= 151646 + 8 else vocab_size - 4
    return {"<|endoftext|>": base, "<|im_start|>": base + 1, "<|im_end|>": base + 2, "<|vision_pad|>": base + 3}


def build_tokenizer(output_dir: str | Path, vocab_size: int = 151936) -> Path:
    """Write tokenizer.json + tokenizer_config.json into ``output_dir``."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers

    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    b2u = _bytes_to_unicode()
    vocab: dict[str, int] = {b2u[b]: b for b in range(256)}
    specials = special_token_ids(vocab_size)
    special_ids = set(specials.values())
    for i in range(256, vocab_size):
        if i in special_ids:
            continue
        text = "".join(b2u[b] for b in f"<t{i}>".encode())
        vocab[text] = i
    for text, idx in specials.items():
        vocab[text] = idx
    model = models.BPE(vocab=vocab, merges=[], fuse_unk=False)
    tok = Tokenizer(model)
    # no merges exist, so every byte is its own token and no split pattern is needed
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)
    tok.decoder = decoders.ByteLevel()
    data = json.loads(tok.to_str())
    data["added_tokens"] = [
        {"id": idx, "content": text, "single_word": False, "lstrip": False, "rstrip": False,
         "normalized": False, "special": True}
        for text, idx in specials.items()
    ]
    (out / "tokenizer.json").write_text(json.dumps(data, ensure_ascii=False), encoding="utf-8")
    config = {
        "tokenizer_class": "PreTrainedTokenizerFast",
        "eos_token": "<|endoftext|>",
        "pad_token": "<|endoftext|>",
        "bos_token": None,
        "unk_token": None,
        "model_max_length": 131072,
        "padding_side": "left",
        "clean_up_tokenization_spaces": False,
        "chat_template": CHAT_TEMPLATE,
        "added_tokens_decoder": {
            str(i): {"content": t, "special": True, "lstrip": False, "rstrip": False, "normalized": False, "single_word": False}
            for t, i in specials.items()
        },
    }
    (out / "tokenizer_config.json").write_text(json.dumps(config, indent=2), encoding="utf-8")
    (out / "special_tokens_map.json").write_text(
        json.dumps({"eos_token": "<|endoftext|>", "pad_token": "<|endoftext|>"}, indent=2), encoding="utf-8"
    )
    return out


def load_tokenizer(path: str | Path):
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(str(path))
    if tok.pad_token_id is None:
        tok.pad_token = tok.eos_token
    tok.padding_side = "left"
    return tok
