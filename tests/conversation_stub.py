"""A tiny tokenizer + Granite-format chat template for Conversation tests (no downloads).

Special tokens ``<|...|>`` are single ids; every other character is one id. The
template renders ``<|start_of_role|>role<|end_of_role|>content<|end_of_text|>``
per message. With ``adapter_name`` an aLoRA adapter's control token replaces
the first token of the generation prompt (its invocation), and a LoRA
adapter's control token is placed at position 0 of the whole render.
"""
import re

_SPECIAL = re.compile(r"<\|[a-zA-Z0-9_\-]+\|>")


class StubTokenizer:
    def __init__(self, adapters: dict[str, str]):
        """``adapters``: name -> "alora" | "lora"."""
        self.adapters = dict(adapters)
        self.specials = ["<|start_of_role|>", "<|end_of_role|>", "<|end_of_text|>"] + [
            f"<|{n}|>" for n in adapters]
        self.special_ids = {s: 10 + i for i, s in enumerate(self.specials)}
        self.id_to_special = {v: k for k, v in self.special_ids.items()}

    def control_token_ids(self):
        return [self.special_ids[f"<|{n}|>"] for n in self.adapters]

    def __call__(self, text, add_special_tokens=False):
        ids = []
        pos = 0
        for m in _SPECIAL.finditer(text):
            ids.extend(1000 + ord(c) for c in text[pos:m.start()])
            ids.append(self.special_ids[m.group(0)])
            pos = m.end()
        ids.extend(1000 + ord(c) for c in text[pos:])
        return {"input_ids": ids}

    def decode(self, ids, skip_special_tokens=True):
        out = []
        for i in ids:
            if i in self.id_to_special:
                if not skip_special_tokens:
                    out.append(self.id_to_special[i])
            else:
                out.append(chr(i - 1000))
        return "".join(out)

    def convert_ids_to_tokens(self, i):
        return self.id_to_special.get(i, chr(i - 1000) if i >= 1000 else None)

    def apply_chat_template(self, messages, add_generation_prompt=False, tokenize=False, adapter_name=None,
                            documents=None, **_):
        parts = []
        if documents:
            parts.append("<|start_of_role|>documents<|end_of_role|>" + "|".join(documents) + "<|end_of_text|>\n")
        for m in messages:
            parts.append(f"<|start_of_role|>{m['role']}<|end_of_role|>{m['content']}<|end_of_text|>\n")
        text = "".join(parts)
        if add_generation_prompt:
            gen = "<|start_of_role|>assistant<|end_of_role|>"
            if adapter_name and self.adapters.get(adapter_name) == "alora":
                gen = f"<|{adapter_name}|>" + gen[len("<|start_of_role|>"):]
            text += gen
        if adapter_name and self.adapters.get(adapter_name) == "lora":
            text = f"<|{adapter_name}|>" + text
        return text


class StubConfig:
    def __init__(self, ids):
        self.adapter_token_ids = list(ids)
