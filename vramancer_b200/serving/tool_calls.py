"""Chat prompt building and tool-call parsing (Hermes `<tool_call>` JSON <-> OpenAI).

* `build_chat_prompt(messages, tools, tool_choice)` — ChatML with a `<tools>` block.
* `parse_tool_calls(text)` — extracts `<tool_call>{...}</tool_call>` blocks (and bare
  JSON objects with name/arguments), repairs common JSON slips (trailing commas,
  single quotes, unbalanced braces), strips `<think>` sections.
* `build_chat_message(text)` — OpenAI assistant message with `tool_calls` and the
  finish reason.
* `detect_tool_loop` — three identical consecutive calls.

Reference parity: core/tool_calls.py:30-207 (parse_tool_calls 60, build_chat_prompt
139, build_chat_message 193).
"""
from __future__ import annotations

import json
import re
import uuid
from typing import Any, Dict, List, Optional, Tuple

_TC_RE = re.compile(r"<tool_call>\s*(.*?)\s*(?:</tool_call>|$)", re.S)
_THINK_RE = re.compile(r"<think>.*?(?:</think>|$)", re.S)


def strip_think(text: str) -> str:
    return _THINK_RE.sub("", text).strip()


def repair_json(s: str) -> Optional[Any]:
    s = s.strip()
    if s.startswith("```"):
        s = s.strip("`")
        s = s[s.find("{"):] if "{" in s else s
    for attempt in range(4):
        try:
            return json.loads(s)
        except json.JSONDecodeError:
            if attempt == 0:
                s = re.sub(r",\s*([}\]])", r"\1", s)            # trailing commas
            elif attempt == 1:
                s = re.sub(r"'", '"', s)                         # single quotes
            elif attempt == 2:
                opens, closes = s.count("{"), s.count("}")
                s = s + "}" * max(0, opens - closes)              # unbalanced braces
    return None


def _normalize(obj: Any) -> Optional[Dict[str, Any]]:
    if not isinstance(obj, dict):
        return None
    if "function" in obj and isinstance(obj["function"], dict):
        obj = obj["function"]
    name = obj.get("name")
    if not name:
        return None
    args = obj.get("arguments", obj.get("parameters", {}))
    if isinstance(args, str):
        parsed = repair_json(args)
        args = parsed if parsed is not None else {"_raw": args}
    return {"name": str(name), "arguments": args}


def parse_tool_calls(text: str) -> Tuple[str, List[Dict[str, Any]]]:
    """Returns (remaining content, [{"name", "arguments"}])."""
    text = strip_think(text)
    calls = []
    for m in _TC_RE.finditer(text):
        c = _normalize(repair_json(m.group(1)))
        if c:
            calls.append(c)
    content = _TC_RE.sub("", text).strip()
    if not calls:
        s = content.strip()
        if s.startswith("{") and '"name"' in s:
            c = _normalize(repair_json(s))
            if c:
                calls.append(c)
                content = ""
    return content, calls


def build_chat_prompt(messages: List[Dict[str, Any]], tools: Optional[List[Dict[str, Any]]] = None,
                      tool_choice: Any = None) -> str:
    parts = []
    sys_msgs = [m for m in messages if m.get("role") == "system"]
    sys_text = "\n".join(str(m.get("content", "")) for m in sys_msgs) or "You are a helpful assistant."
    if tools and tool_choice != "none":
        specs = "\n".join(json.dumps(t.get("function", t)) for t in tools)
        sys_text += ("\n\n# Tools\n\nYou may call one or more functions to assist with the user query.\n"
                     f"<tools>\n{specs}\n</tools>\n\nFor each function call, return a json object with function "
                     "name and arguments within <tool_call></tool_call> XML tags.")
        if isinstance(tool_choice, dict) and tool_choice.get("function"):
            sys_text += f"\nYou must call the function {tool_choice['function'].get('name')}."
        elif tool_choice == "required":
            sys_text += "\nYou must call at least one function."
    parts.append(f"<|im_start|>system\n{sys_text}<|im_end|>")
    for m in messages:
        role = m.get("role")
        if role == "system":
            continue
        content = m.get("content") or ""
        if isinstance(content, list):
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        if role == "assistant" and m.get("tool_calls"):
            calls = "".join(f"<tool_call>\n{json.dumps(tc.get('function', tc))}\n</tool_call>"
                            for tc in m["tool_calls"])
            content = (content + "\n" + calls).strip()
        if role == "tool":
            parts.append(f"<|im_start|>user\n<tool_response>\n{content}\n</tool_response><|im_end|>")
            continue
        parts.append(f"<|im_start|>{role}\n{content}<|im_end|>")
    parts.append("<|im_start|>assistant\n")
    return "\n".join(parts)


def build_chat_message(text: str) -> Tuple[Dict[str, Any], str]:
    content, calls = parse_tool_calls(text)
    msg: Dict[str, Any] = {"role": "assistant", "content": content or None}
    if calls:
        msg["tool_calls"] = [{"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                              "function": {"name": c["name"], "arguments": json.dumps(c["arguments"])}}
                             for c in calls]
        return msg, "tool_calls"
    if msg["content"] is None:
        msg["content"] = ""
    return msg, "stop"


def detect_tool_loop(history: List[Dict[str, Any]], repeats: int = 3) -> bool:
    calls = []
    for m in history:
        for tc in m.get("tool_calls") or []:
            f = tc.get("function", tc)
            calls.append((f.get("name"), json.dumps(f.get("arguments"), sort_keys=True)
                          if not isinstance(f.get("arguments"), str) else f.get("arguments")))
    return len(calls) >= repeats and len(set(calls[-repeats:])) == 1
