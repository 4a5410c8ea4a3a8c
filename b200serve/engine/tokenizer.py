"""Tokenizers: an HF tokenizer when the model directory ships one, else a
self-contained synthetic tokenizer for random-init shapes.

The synthetic tokenizer maps UTF-8 bytes to ids 3..258 and renders a ChatML
template ("<|im_start|>role\\ncontent<|im_end|>\\n" + assistant header, with
"<think>\\n" pre-filled when thinking is on, as Qwen templates do). Ids outside
the byte range decode to a short placeholder word so random-weight models
still stream readable text.
"""

from __future__ import annotations


class SyntheticTokenizer:
    BYTE0 = 3

    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size
        self.im_start_id = vocab_size - 3
        self.im_end_id = vocab_size - 2
        self.eos_token_id = vocab_size - 1
        self.pad_token_id = self.eos_token_id
        self._special = {self.im_start_id: "<|im_start|>", self.im_end_id: "<|im_end|>",
                         self.eos_token_id: "<|endoftext|>"}
        self._by_text = {}

    def add_special(self, tokens: dict):
        """Map marker strings to ids ({"<|image_pad|>": id, ...}) for encode and decode."""
        for text, i in tokens.items():
            self._special[int(i)] = text
            self._by_text[text] = int(i)

    def encode(self, text: str, add_special_tokens: bool = False) -> list:
        if not self._by_text:
            return [b + self.BYTE0 for b in text.encode("utf-8")]
        out, i = [], 0
        while i < len(text):
            hit = next((t for t in self._by_text if text.startswith(t, i)), None)
            if hit is not None:
                out.append(self._by_text[hit])
                i += len(hit)
                continue
            out += [b + self.BYTE0 for b in text[i].encode("utf-8")]
            i += 1
        return out

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out = bytearray()
        words = []
        for i in ids:
            i = int(i)
            if self.BYTE0 <= i < self.BYTE0 + 256:
                out.append(i - self.BYTE0)
            elif i in self._special:
                if not skip_special_tokens:
                    out.extend(self._special[i].encode())
            else:
                out.extend(f" w{i % 9973}".encode())
        del words
        return out.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, add_generation_prompt=True, enable_thinking=True, tools=None,
                            **_) -> list:
        ids = []
        if tools:
            from b200serve.core.tool_calls import tools_system_block
            messages = [{"role": "system", "content": tools_system_block(tools)}] + list(messages)
        for m in messages:
            content = m.get("content", "")
            if isinstance(content, list):
                content = "\n".join(p.get("text", "") for p in content if isinstance(p, dict))
            ids += [self.im_start_id] + self.encode(f"{m.get('role', 'user')}\n{content}") + [self.im_end_id]
            ids += self.encode("\n")
        if add_generation_prompt:
            ids += [self.im_start_id] + self.encode("assistant\n")
            if enable_thinking:
                ids += self.encode("<think>\n")
        return ids

    @property
    def stop_ids(self) -> set:
        return {self.im_end_id, self.eos_token_id}


class HFTokenizer:
    """Wraps a transformers tokenizer behind the same small interface."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer
        from b200serve.core.config import TRUST_REMOTE_CODE
        self.tok = AutoTokenizer.from_pretrained(path, trust_remote_code=TRUST_REMOTE_CODE)
        self.vocab_size = len(self.tok)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text, add_special_tokens=False):
        return self.tok.encode(text, add_special_tokens=add_special_tokens)

    def decode(self, ids, skip_special_tokens=True):
        return self.tok.decode(ids, skip_special_tokens=skip_special_tokens)

    def apply_chat_template(self, messages, add_generation_prompt=True, enable_thinking=True, tools=None, **_):
        kw = {"tools": tools} if tools else {}
        try:
            out = self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                               enable_thinking=enable_thinking, tokenize=True, **kw)
        except TypeError:
            out = self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt, tokenize=True,
                                               **kw)
        if isinstance(out, dict) or hasattr(out, "input_ids"):    # BatchEncoding from newer tokenizers
            out = out["input_ids"]
        return list(out)

    @property
    def stop_ids(self) -> set:
        s = set()
        if self.eos_token_id is not None:
            s |= set(self.eos_token_id) if isinstance(self.eos_token_id, list) else {self.eos_token_id}
        for name in ("<|im_end|>", "<|endoftext|>"):
            i = self.tok.convert_tokens_to_ids(name)
            if i is not None and i != getattr(self.tok, "unk_token_id", None):
                s.add(i)
        return s


def load_tokenizer(model_path, vocab_size):
    import os
    if model_path and os.path.isdir(model_path) and any(
            os.path.exists(os.path.join(model_path, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        return HFTokenizer(model_path)
    return SyntheticTokenizer(vocab_size)


class IncrementalDecoder:
    """Turns a growing id list into text deltas without splitting UTF-8 sequences."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids = []
        self.text = ""

    def push(self, token_id: int) -> str:
        self.ids.append(int(token_id))
        full = self.tok.decode(self.ids)
        if full.endswith("�"):
            return ""  # wait for the rest of a multi-byte character
        delta = full[len(self.text):]
        self.text = full
        return delta
