"""Tokenizers of the engine's text API and the HTTP server.

``ByteTokenizer`` (random-weight models): UTF-8 bytes are token ids 0..255,
ids >= 256 decode to nothing. ``HFTokenizer``: a checkpoint directory's own
tokenizer through transformers (local files only), with its chat template.
"""


def render_chat(template: str, messages) -> str:
    """A Jinja chat template (the format of Hugging Face ``chat_template``)
    rendered for ``messages`` with the generation prompt appended, in a
    sandboxed environment."""
    from jinja2.sandbox import ImmutableSandboxedEnvironment

    env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
    return env.from_string(template).render(messages=messages, add_generation_prompt=True)


def load_chat_template(arg: str) -> str:
    """``--chat-template``: a file path, else the template text itself."""
    import os

    if os.path.isfile(arg):
        with open(arg) as f:
            return f.read()
    return arg


class ByteTokenizer:
    """UTF-8 bytes as token ids (ids >= 256 have no text)."""

    def __init__(self, chat_template: str = None):
        self.chat_template = chat_template

    def encode(self, text: str) -> list:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def chat(self, messages) -> list:
        if self.chat_template:
            return self.encode(render_chat(self.chat_template, messages))
        text = "".join(f"<|{m.get('role', 'user')}|>{m.get('content', '')}" for m in messages) + "<|assistant|>"
        return self.encode(text)


class HFTokenizer:
    """A checkpoint directory's tokenizer (transformers, local files only)."""

    # one of these must be present: given only config.json, transformers 5
    # builds an empty tokenizer that maps all text to <unk>
    FILES = ("tokenizer.json", "tokenizer.model", "vocab.json", "tokenizer_config.json")

    def __init__(self, path: str, chat_template: str = None):
        import os

        from transformers import AutoTokenizer

        if os.path.isdir(path) and not any(os.path.isfile(os.path.join(path, f)) for f in self.FILES):
            raise FileNotFoundError(f"no tokenizer files in {path} (looked for {', '.join(self.FILES)})")
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        if chat_template:  # replaces the checkpoint's own template
            self.tok.chat_template = chat_template

    def encode(self, text: str) -> list:
        return self.tok.encode(text, add_special_tokens=True)

    def decode(self, ids) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def chat(self, messages) -> list:
        if getattr(self.tok, "chat_template", None):
            r = self.tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True)
            if hasattr(r, "keys"):  # transformers 5 returns a BatchEncoding, 4 a list of ids
                r = r["input_ids"]
            return [int(t) for t in r]
        return self.encode("".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in messages))
