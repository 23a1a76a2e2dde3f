"""A character-level tokenizer with Granite's role markers as special tokens (no network needed).

Every character is one token except the markers (special) and a few added
words (``<think>``, ``</think>``, ``<requirements``) that make multi-character
tokens, as real Granite tokenizers have.
"""
from __future__ import annotations

import os

MARKERS = ["<|start_of_role|>", "<|end_of_role|>", "<|end_of_text|>", "<|im_start|>", "<|im_end|>",
           "<|unused_0|>", "<|unused_1|>"]
WORDS = ["<think>", "</think>", "<requirements"]
FIXTURES = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fixtures", "chat_templates")


def make_tokenizer(template: str | None = None):
    from tokenizers import AddedToken, Regex, Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {"<unk>": 0}
    for c in [chr(i) for i in range(32, 127)] + ["\n", "\t"]:
        vocab.setdefault(c, len(vocab))
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Split(Regex(r"[\s\S]"), behavior="isolated")
    tok.decoder = decoders.Fuse()
    tok.add_special_tokens([AddedToken(t, special=True, normalized=False) for t in MARKERS])
    tok.add_tokens([AddedToken(t, normalized=False) for t in WORDS])
    t = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>")
    if template is not None:
        t.chat_template = template
    return t


def granite_template(version: str) -> str:
    with open(os.path.join(FIXTURES, f"granite-{version}.jinja")) as f:
        return f.read()
