"""Tokenizers for the server: a local Hugging Face tokenizer, or a byte tokenizer.

With a checkpoint directory the server loads its tokenizer (offline,
``transformers.AutoTokenizer``) and its chat template.  Without one (random
weights, benchmarks) :class:`ByteTokenizer` maps UTF-8 bytes to ids
``BYTE0..BYTE0+255`` and renders every other id as ``<id>``, so each generated
token is one non-empty text piece and a streaming client counts tokens by
chunks, as the sweep client does.
"""

from __future__ import annotations


class ByteTokenizer:
    BYTE0 = 16

    def __init__(self, vocab_size: int, bos_id: int = 0, eos_id: int = 1):
        self.vocab_size = vocab_size
        self.bos_token_id = bos_id
        self.eos_token_id = eos_id

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [self.BYTE0 + b for b in text.encode("utf-8")]
        return ([self.bos_token_id] if add_bos else []) + ids

    def decode_token(self, tid: int) -> str:
        if self.BYTE0 <= tid < self.BYTE0 + 256:
            b = tid - self.BYTE0
            return chr(b) if b < 128 else f"<0x{b:02X}>"
        return f"<{tid}>"

    def decode(self, ids: list[int]) -> str:
        out, buf = [], bytearray()
        for t in ids:
            if self.BYTE0 <= t < self.BYTE0 + 256:
                buf.append(t - self.BYTE0)
                continue
            if buf:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
            if t not in (self.bos_token_id, self.eos_token_id):
                out.append(f"<{t}>")
        if buf:
            out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)

    def apply_chat_template(self, messages: list[dict]) -> str:
        return render_chat(messages)

    def stream_decoder(self) -> "PieceDecoder":
        """One text piece per token (the benchmark clients count tokens by chunks)."""
        return PieceDecoder(self)


class PieceDecoder:
    """Streaming text of a token sequence, one token's own text per token."""

    def __init__(self, tok):
        self.tok = tok

    def push(self, tid: int) -> str:
        return self.tok.decode_token(tid)

    def flush(self) -> str:
        return ""


class IncrementalDecoder:
    """Streaming text of a token sequence for tokenizers whose tokens are not whole
    characters (byte-level BPE): each token's delta is the new text of the decoded
    window ``ids[prefix:]`` beyond the text of ``ids[prefix:read]``, and a delta
    that would end in U+FFFD (a character whose bytes are still arriving) is held
    back until a later token completes it.  Decoding a short window keeps the
    tokenizer's context-dependent rules (leading spaces, merges) right at its
    edge.  This is the incremental detokenization that text-generation servers
    use (Hugging Face ``TextStreamer``, vLLM's ``detokenize_incrementally``)."""

    def __init__(self, decode):
        self.decode = decode          # list[int] -> str
        self.ids: list[int] = []
        self.prefix = 0
        self.read = 0

    def push(self, tid: int) -> str:
        self.ids.append(tid)
        before = self.decode(self.ids[self.prefix:self.read])
        now = self.decode(self.ids[self.prefix:])
        if len(now) > len(before) and not now.endswith("\ufffd"):
            self.prefix, self.read = self.read, len(self.ids)
            return now[len(before):]
        return ""

    def flush(self) -> str:
        """Text still held back at the end of the sequence (an incomplete character
        comes out as U+FFFD)."""
        before = self.decode(self.ids[self.prefix:self.read])
        now = self.decode(self.ids[self.prefix:])
        self.prefix = self.read = len(self.ids)
        return now[len(before):]


def render_chat(messages: list[dict]) -> str:
    """DeepSeek-style chat rendering used when the tokenizer has no template."""
    parts = []
    for m in messages:
        role, content = m.get("role", "user"), m.get("content", "")
        if isinstance(content, list):  # OpenAI content parts
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        if role == "system":
            parts.append(content)
        elif role == "user":
            parts.append(f"<｜User｜>{content}")
        else:
            parts.append(f"<｜Assistant｜>{content}<｜end▁of▁sentence｜>")
    parts.append("<｜Assistant｜>")
    return "".join(parts)


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True, trust_remote_code=False)
        self.bos_token_id = self.tok.bos_token_id
        self.eos_token_id = self.tok.eos_token_id
        self.vocab_size = len(self.tok)

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = self.tok.encode(text, add_special_tokens=False)
        return ([self.bos_token_id] if add_bos and self.bos_token_id is not None else []) + ids

    def decode_token(self, tid: int) -> str:
        return self.tok.decode([tid])

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def stream_decoder(self) -> IncrementalDecoder:
        return IncrementalDecoder(self.decode)

    def apply_chat_template(self, messages: list[dict]) -> str:
        if getattr(self.tok, "chat_template", None):
            return self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
        return render_chat(messages)


def load_tokenizer(path: str | None, cfg):
    if path:
        return HFTokenizer(path)
    return ByteTokenizer(cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
