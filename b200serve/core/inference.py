"""Backend-agnostic text and context utilities (reference: core/inference.py).

* ``ThinkFilter`` splits a token stream into thinking and answer text
  (reference :28-94): the stream may start inside ``<think>``; ``</think>``
  (Qwen) or ``<channel|>`` (Gemma 4) closes a thinking block, ``<think>``
  opens one. A tail of the buffer is held back so a tag split across two
  chunks is still recognised.
* ``strip_think_blocks`` / ``_clean_response`` / ``_truncate_repetition``
  clean a finished answer (reference :97-191).
* ``context_input_budget`` / ``ensure_context_fit`` / ``compress_history`` /
  ``trim_messages_to_context`` / ``plan_compaction`` keep a conversation
  inside the engine's context window (reference :297-720).
"""

from __future__ import annotations

import logging
import re

_log = logging.getLogger(__name__)

STOP_STRINGS = [
    "\nUser:", "\nUSER:", "\nYOU:", "\nuser:", "\nHuman:",
    "\nuser\n", "\nUser\n", "\nassistant\n", "\nassistant ",
    "\n<end_of_turn>", "<end_of_turn>",
    "\n[TOOL OUTPUT", "\n[tool output",
]

_THINK_OPEN = "<think>"
_THINK_CLOSERS = ("</think>", "<channel|>")


class ThinkFilter:
    """Route streamed text to ``on_thinking`` or ``on_response``.

    feed() may be called with arbitrary fragments; flush() emits whatever is
    still held back once the stream ends.
    """

    # Longest tag that can be pending in each state: in thinking mode the
    # closers (up to 10 chars), in answer mode the opener (7 chars).
    _HOLD_THINK = max(len(t) for t in _THINK_CLOSERS)
    _HOLD_ANSWER = len(_THINK_OPEN)

    def __init__(self, on_response, on_thinking=None, starts_in_think=True):
        self.on_response = on_response
        self.on_thinking = on_thinking
        self.in_think = starts_in_think
        self.buffer = ""

    def feed(self, text):
        self.buffer += text
        while self._step():
            pass

    def _first_closer(self):
        best = (-1, 0)
        for tag in _THINK_CLOSERS:
            i = self.buffer.find(tag)
            if i != -1 and (best[0] == -1 or i < best[0]):
                best = (i, len(tag))
            if i != -1 and tag == _THINK_CLOSERS[0]:
                # "</think>" wins whenever present, as in the reference
                return i, len(tag)
        return best

    def _step(self) -> bool:
        """Consume what can be decided now; True if the state changed."""
        if self.in_think:
            idx, n = self._first_closer()
            if idx != -1:
                if self.on_thinking and idx > 0:
                    self.on_thinking(self.buffer[:idx])
                self.buffer = self.buffer[idx + n:]
                self.in_think = False
                return True
            if self.on_thinking and len(self.buffer) > self._HOLD_THINK:
                cut = len(self.buffer) - self._HOLD_THINK
                self.on_thinking(self.buffer[:cut])
                self.buffer = self.buffer[cut:]
            return False
        idx = self.buffer.find(_THINK_OPEN)
        if idx != -1:
            if idx > 0:
                self.on_response(self.buffer[:idx])
            self.buffer = self.buffer[idx + len(_THINK_OPEN):]
            self.in_think = True
            return True
        if len(self.buffer) > self._HOLD_ANSWER:
            cut = len(self.buffer) - self._HOLD_ANSWER
            self.on_response(self.buffer[:cut])
            self.buffer = self.buffer[cut:]
        return False

    def flush(self):
        if self.buffer:
            if not self.in_think:
                self.on_response(self.buffer)
            elif self.on_thinking:
                self.on_thinking(self.buffer)
        self.buffer = ""


def strip_think_blocks(text: str) -> str:
    """Remove ``<think>...</think>`` pairs, and a leading unpaired thinking
    prefix (text that starts mid-thought and is closed by ``</think>`` before
    any ``<think>``)."""
    text = re.sub(r"<think>.*?</think>", "", text, flags=re.DOTALL)
    close = text.find("</think>")
    if close != -1:
        opener = text.find("<think>")
        if opener == -1 or close < opener:
            text = text[close + len("</think>"):]
    return text.strip()


def _truncate_repetition(text: str, min_phrase_len: int = 80) -> str:
    """Cut a verbatim loop: 3+ back-to-back copies of an 80+ char phrase whose
    gaps are each under a quarter of the phrase length. Structured output
    with data between repeated boilerplate is left alone."""
    if len(text) < min_phrase_len * 4:
        return text
    for plen in range(min_phrase_len, min(500, len(text) // 3) + 1, 20):
        gap = plen // 4
        for start in range(0, len(text) - plen * 3):
            phrase = text[start:start + plen]
            end1 = start + plen
            second = text.find(phrase, end1, end1 + gap + plen)
            if second == -1:
                continue
            end2 = second + plen
            if text.find(phrase, end2, end2 + gap + plen) == -1:
                continue
            return text[:second].rstrip()
    return text


def _clean_response(text: str, stop_strings: bool = True) -> str:
    clean = strip_think_blocks(text)
    if stop_strings:
        for marker in STOP_STRINGS:
            i = clean.find(marker)
            if i != -1:
                clean = clean[:i]
    return _truncate_repetition(clean).rstrip()


# ----- token counting -----
_tokenizer = None  # set by engines after load for exact counts


def _flatten_for_count(content) -> str:
    if isinstance(content, str):
        return content
    if not isinstance(content, list):
        return ""
    parts = []
    for p in content:
        if isinstance(p, str):
            parts.append(p)
        elif isinstance(p, dict) and p.get("type") == "text":
            parts.append(p.get("text", "") or "")
    return "\n".join(parts)


def _count_image_parts(messages) -> int:
    n = 0
    for m in messages:
        c = m.get("content")
        if isinstance(c, list):
            n += sum(1 for p in c if isinstance(p, dict)
                     and p.get("type") in ("image_url", "image", "input_image"))
    return n


def _count_tokens(messages, tokenizer=None) -> int:
    from b200serve.core.request_estimator import TOKENS_PER_IMAGE
    img = _count_image_parts(messages) * TOKENS_PER_IMAGE
    tok = tokenizer or _tokenizer
    if tok is not None:
        text = "\n".join(_flatten_for_count(m.get("content")) for m in messages)
        return len(tok.encode(text, add_special_tokens=False)) + img
    return sum(len(_flatten_for_count(m.get("content"))) for m in messages) // 4 + img


def _extract_key_point(msg) -> str:
    content = msg.get("content") if isinstance(msg.get("content"), str) else _flatten_for_count(msg.get("content"))
    if content.startswith("[TOOL OUTPUT") or content.startswith("[TOOL RESULT"):
        lines = [l.strip() for l in content.split("\n") if l.strip()]
        for prefix, fmt in (("File:", "Read: {}"), ("Found ", "{}")):
            for l in lines:
                if l.startswith(prefix):
                    return fmt.format(l[:120])
        return lines[0][:80] if lines else "(tool output)"
    if msg.get("role") == "user":
        return content.split("\n")[0].strip()[:100]
    for s in re.split(r"[.!?\n]", content):
        s = s.strip().lstrip("#*- ")
        if len(s) > 15:
            return s[:100]
    return content[:100]


def context_input_budget(engine_ctx: int, max_tokens, floor_frac: float = 0.25) -> int:
    """Input tokens that still leave room for ``max_tokens`` of completion and
    a template margin of max(512, ctx/32); never below ``floor_frac`` of ctx."""
    if engine_ctx <= 0:
        return 0
    margin = max(512, engine_ctx // 32)
    return max(engine_ctx - int(max_tokens or 0) - margin, int(engine_ctx * floor_frac))


def compress_history(history, context_window):
    """Fold all but the newest ``context_window - 1`` messages into one
    key-point summary; the system prompt and the first user message (the
    original task) are kept verbatim."""
    convo = history[1:]
    if len(convo) <= context_window:
        return list(history)
    pinned = convo[0] if convo and convo[0].get("role") == "user" else None
    rest = convo[1:] if pinned else convo
    keep = max(context_window - 1, 1)
    if len(rest) <= keep:
        return list(history)
    old, recent = rest[:-keep], rest[-keep:]
    points = [("Q" if m.get("role") == "user" else "A") + ": " + _extract_key_point(m) for m in old]
    out = [history[0]]
    if pinned:
        out.append(pinned)
    out.append({"role": "user", "content": "[EARLIER CONVERSATION — key points]\n" + "\n".join(points)})
    out.extend(recent)
    return out


def trim_messages_to_context(messages, max_input_tokens):
    """Drop the oldest middle messages until under budget; keep the system
    prompt and the last two messages, truncating the last one if needed."""
    if max_input_tokens <= 0 or len(messages) <= 1 or _count_tokens(messages) <= max_input_tokens:
        return messages
    system = messages[:1]
    middle = list(messages[1:-2]) if len(messages) > 3 else []
    tail = list(messages[-2:]) if len(messages) >= 2 else []
    while middle and _count_tokens(system + middle + tail) > max_input_tokens:
        middle.pop(0)
    result = system + middle + tail
    over = _count_tokens(result) - max_input_tokens
    if over > 0 and len(result) >= 2:
        last = dict(result[-1])
        content = last.get("content", "")
        if isinstance(content, str):
            cut = over * 4 + 200
            if cut < len(content):
                last["content"] = content[:len(content) - cut] + "\n[...trimmed...]"
                result[-1] = last
    return result


def ensure_context_fit(messages, engine_ctx, max_tokens, context_window=15, count_fn=None):
    """Guarantee ``messages`` plus ``max_tokens`` of completion fit ``engine_ctx``:
    compact, then hard-trim, then re-check against an exact counter when given.
    Returns (messages, {"budget", "est", "compacted", "trimmed"})."""
    info = {"budget": 0, "est": 0, "compacted": False, "trimmed": False}
    if engine_ctx <= 0 or not messages:
        return messages, info
    budget = context_input_budget(engine_ctx, max_tokens)
    info["budget"] = budget
    est = _count_tokens(messages)
    if est > budget and len(messages) > 4:
        compacted = compress_history(messages, min(max(budget // 500, context_window), 200))
        if len(compacted) < len(messages):
            messages, info["compacted"] = compacted, True
        est = _count_tokens(messages)
    if est > budget:
        messages, info["trimmed"] = trim_messages_to_context(messages, budget), True
        est = _count_tokens(messages)
    if count_fn is not None:
        text = "\n".join(m.get("content", "") for m in messages if isinstance(m.get("content"), str))
        try:
            exact = count_fn(text)
        except Exception:
            exact = 0
        if exact and exact > budget:
            adjusted = max(int(budget * max(est, 1) / exact), 256)
            messages, info["trimmed"] = trim_messages_to_context(messages, adjusted), True
            est = _count_tokens(messages)
    info["est"] = est
    return messages, info


def auto_compact_if_needed(messages, engine_ctx, context_window, threshold=0.60):
    if engine_ctx <= 0 or len(messages) <= 4:
        return messages, False
    limit = int(engine_ctx * threshold)
    if _count_tokens(messages) <= limit:
        return messages, False
    return compress_history(messages, min(max(limit // 500, context_window), 200)), True


COMPACT_HIGH = 0.80
COMPACT_TARGET = 0.10
COMPACT_MAX_MESSAGES = 160
COMPACT_KEEP_MAX = 20
COMPACT_TAG = "[EARLIER CONVERSATION — AUTO-COMPACTED SUMMARY]"


def _is_compact_summary(msg) -> bool:
    return (msg.get("role") == "user" and isinstance(msg.get("content"), str)
            and msg["content"].startswith("[EARLIER CONVERSATION"))


def plan_compaction(messages, engine_ctx, max_tokens, high=COMPACT_HIGH,
                    target=COMPACT_TARGET, max_messages=COMPACT_MAX_MESSAGES) -> int:
    """Number of leading conversation messages to fold (0 = not due)."""
    convo = messages[1:]
    if engine_ctx <= 0 or len(convo) < 4:
        return 0
    budget = context_input_budget(engine_ctx, max_tokens)
    if _count_tokens(messages) <= budget * high and len(convo) <= max_messages:
        return 0
    kept, used = 0, 0
    for msg in reversed(convo):
        if _is_compact_summary(msg):
            break
        cost = _count_tokens([msg])
        if kept >= 2 and (used + cost > budget * target or kept >= COMPACT_KEEP_MAX):
            break
        kept += 1
        used += cost
    cut = len(convo) - kept
    if cut < 1 or (cut == 1 and _is_compact_summary(convo[0])):
        return 0
    return cut


def extractive_synopsis(head) -> str:
    pts = []
    for m in head:
        if _is_compact_summary(m):
            pts.append(m["content"].split("\n", 1)[-1].strip())
        else:
            pts.append(("Q" if m.get("role") == "user" else "A") + ": " + _extract_key_point(m))
    return "\n".join(pts)


def apply_compaction(messages, cut, synopsis):
    return ([messages[0], {"role": "user", "content": f"{COMPACT_TAG}\n{synopsis.strip()}"}]
            + list(messages[1 + cut:]))


def check_vram_pressure(threshold=0.85):
    """(pressured, fraction, allocated_gb, total_gb) for the current device."""
    try:
        import torch
        if not torch.cuda.is_available():
            return False, 0.0, 0.0, 0.0
        free, total = torch.cuda.mem_get_info()
        used = total - free
        frac = used / total
        return frac >= threshold, frac, used / 1e9, total / 1e9
    except Exception:
        return False, 0.0, 0.0, 0.0
