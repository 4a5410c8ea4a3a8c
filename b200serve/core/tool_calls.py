"""OpenAI-style function calling for chat models that emit Hermes/Qwen tool-call blocks.

The request's ``tools`` go into the chat template (the model's own template when the
checkpoint has one; otherwise a system block that lists them). The model answers a call
as ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``; those blocks are taken out
of the visible text and returned as ``tool_calls`` with ``finish_reason`` "tool_calls".
Reference behaviour: the API's tool loop and ``x_tool_status`` events (api/server.py:1218-1571),
which run the reference's own server-side tools; here the calls go back to the client, as
in the OpenAI API.
"""

from __future__ import annotations

import json
import re
import uuid

OPEN, CLOSE = "<tool_call>", "</tool_call>"
_BLOCK = re.compile(r"<tool_call>\s*(.*?)\s*</tool_call>", re.S)


def tools_system_block(tools) -> str:
    """A system message that lists ``tools`` for templates without tool support."""
    lines = ["# Tools", "", "You may call one or more functions. Function signatures:", "<tools>"]
    lines += [json.dumps(t, ensure_ascii=False) for t in tools]
    lines += ["</tools>", "",
              "For each call, return a JSON object with the function name and arguments inside "
              "<tool_call></tool_call> tags."]
    return "\n".join(lines)


def parse(text: str):
    """(visible text, tool_calls list) from a completion."""
    calls = []
    for m in _BLOCK.finditer(text):
        try:
            obj = json.loads(m.group(1))
        except ValueError:
            continue
        if not isinstance(obj, dict) or "name" not in obj:
            continue
        args = obj.get("arguments", obj.get("parameters", {}))
        calls.append({"id": "call_" + uuid.uuid4().hex[:12], "type": "function",
                      "function": {"name": str(obj["name"]),
                                   "arguments": args if isinstance(args, str) else json.dumps(args)}})
    visible = _BLOCK.sub("", text).strip() if calls else text
    return visible, calls


class ToolCallFilter:
    """Streaming filter: passes text outside tool-call blocks to ``on_text`` and keeps the
    blocks; ``finish()`` returns the parsed calls."""

    def __init__(self, on_text):
        self.on_text = on_text
        self.buf = ""
        self.inside = False
        self.raw = ""

    def feed(self, piece: str):
        self.buf += piece
        while self.buf:
            if self.inside:
                i = self.buf.find(CLOSE)
                if i < 0:
                    return
                self.raw += OPEN + self.buf[:i + len(CLOSE)]
                self.buf = self.buf[i + len(CLOSE):]
                self.inside = False
            else:
                i = self.buf.find(OPEN)
                if i >= 0:
                    if i:
                        self.on_text(self.buf[:i])
                    self.buf = self.buf[i + len(OPEN):]
                    self.inside = True
                    continue
                keep = 0          # hold back a possible partial "<tool_call>" at the end
                for k in range(min(len(OPEN) - 1, len(self.buf)), 0, -1):
                    if OPEN.startswith(self.buf[-k:]):
                        keep = k
                        break
                if len(self.buf) > keep:
                    self.on_text(self.buf[:len(self.buf) - keep])
                    self.buf = self.buf[len(self.buf) - keep:]
                return

    def finish(self):
        if self.buf and not self.inside:
            self.on_text(self.buf)
        self.buf = ""
        return parse(self.raw)[1]
