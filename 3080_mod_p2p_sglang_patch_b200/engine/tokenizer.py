"""Tokenizers of the engine's text API and the HTTP server.

``ByteTokenizer`` (random-weight models): UTF-8 bytes are token ids 0..255,
ids >= 256 decode to nothing. ``HFTokenizer``: a checkpoint directory's own
tokenizer through transformers (local files only), with its chat template.
"""


class ByteTokenizer:
    """UTF-8 bytes as token ids (ids >= 256 have no text)."""

    def encode(self, text: str) -> list:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")


class HFTokenizer:
    """A checkpoint directory's tokenizer (transformers, local files only)."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)

    def encode(self, text: str) -> list:
        return self.tok.encode(text, add_special_tokens=True)

    def decode(self, ids) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def chat(self, messages) -> list:
        if getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True))
        return self.encode("".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in messages))
