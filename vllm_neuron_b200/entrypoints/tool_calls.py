"""Tool calling for the OpenAI chat endpoint.

Behaviour of the Trainium plugin's serving stack (``docs/guides/features-guide.md:654-690``,
vLLM's tool-calling front end): two paths by ``tool_choice``:

* ``"required"`` or a named function: the tool schemas become a JSON-schema constraint that
  runs through the structured-output bitmask like any ``response_format``.  ``required``
  generates ``[{"name": <one of the tools>, "parameters": {...}}, ...]``; a named function
  generates that function's arguments object directly (both as compact JSON, without free
  whitespace);
* ``"auto"``: no constraint; after generation a parser extracts calls from the text.  The
  parsers cover the formats GPT-OSS and common chat templates emit: harmony messages to
  ``functions.<name>`` (``<|channel|>commentary to=functions.f ... <|message|>{...}<|call|>``),
  Hermes ``<tool_call>{...}</tool_call>`` blocks and a bare JSON object / list with ``name``
  and ``arguments`` (or ``parameters``);
* ``"none"`` (or no tools): plain chat.

Responses carry ``message.tool_calls`` (``id``, ``type: function``, ``function.name``,
``function.arguments`` as a JSON string), ``content`` holds the text outside the calls, and
``finish_reason`` is ``"tool_calls"`` when any call was produced.
"""

from __future__ import annotations

import json
import re
import uuid
from typing import Any

PARSERS = ("auto", "openai", "hermes", "json")


class ToolChoiceError(ValueError):
    pass


def _functions(tools: list[dict] | None) -> dict[str, dict]:
    out = {}
    for t in tools or []:
        if t.get("type", "function") != "function" or "function" not in t:
            raise ToolChoiceError(f"unsupported tool entry: {t!r}")
        f = t["function"]
        if not f.get("name"):
            raise ToolChoiceError("every function needs a name")
        out[f["name"]] = f.get("parameters") or {"type": "object", "properties": {}}
    return out


def named_choice(tool_choice: Any) -> str | None:
    if isinstance(tool_choice, dict):
        return (tool_choice.get("function") or {}).get("name")
    return None


def tool_constraint(tools: list[dict] | None, tool_choice: Any) -> dict | None:
    """The structured-output constraint a ``tool_choice`` implies (None: unconstrained)."""
    fns = _functions(tools)
    if not fns or tool_choice in (None, "auto", "none"):
        return None
    name = named_choice(tool_choice)
    if name is not None:
        if name not in fns:
            raise ToolChoiceError(f"tool_choice names unknown function {name!r}")
        return {"json": fns[name], "disable_any_whitespace": True}
    if tool_choice != "required":
        raise ToolChoiceError(f"unsupported tool_choice {tool_choice!r}")
    items = [{"type": "object",
              "properties": {"name": {"type": "string", "enum": [n]}, "parameters": p},
              "required": ["name", "parameters"]} for n, p in fns.items()]
    return {"json": {"type": "array", "minItems": 1,
                     "items": items[0] if len(items) == 1 else {"anyOf": items}},
            "disable_any_whitespace": True}


def _call(name: str, args: Any) -> dict:
    return {"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
            "function": {"name": name, "arguments": args if isinstance(args, str) else json.dumps(args)}}


_HARMONY = re.compile(r"to=functions\.([\w\-\.]+)[^<]*(?:<\|constrain\|>\s*\w+\s*)?<\|message\|>(.*?)(?:<\|call\|>|<\|end\|>|$)",
                      re.S)
_HERMES = re.compile(r"<tool_call>\s*(.*?)\s*</tool_call>", re.S)


def _from_obj(obj: Any, known: set[str]) -> list[dict]:
    objs = obj if isinstance(obj, list) else [obj]
    calls = []
    for o in objs:
        if not isinstance(o, dict):
            return []
        name = o.get("name")
        args = o.get("arguments", o.get("parameters", {}))
        if not isinstance(name, str) or (known and name not in known):
            return []
        calls.append(_call(name, args))
    return calls


def parse_tool_calls(text: str, tools: list[dict] | None, parser: str = "auto") -> tuple[str | None, list[dict]]:
    """Tool calls in generated ``text``: (remaining content or None, calls)."""
    known = set(_functions(tools))
    if parser in ("auto", "openai"):
        hits = list(_HARMONY.finditer(text))
        if hits:
            calls = []
            for m in hits:
                body = m.group(2).strip()
                try:
                    args = json.loads(body)
                except ValueError:
                    args = body
                if not known or m.group(1) in known:
                    calls.append(_call(m.group(1), args))
            # the text before the call, without the harmony header that opens the call message
            content = re.split(r"<\|(?:start|channel)\|>", text[:hits[0].start()])[0].strip()
            if calls:
                return (content or None), calls
    if parser in ("auto", "hermes"):
        hits = list(_HERMES.finditer(text))
        if hits:
            calls = []
            for m in hits:
                try:
                    calls += _from_obj(json.loads(m.group(1)), known)
                except ValueError:
                    continue
            if calls:
                content = _HERMES.sub("", text).strip()
                return (content or None), calls
    if parser in ("auto", "json"):
        s = text.strip()
        if s[:1] in "[{":
            try:
                calls = _from_obj(json.loads(s), known)
            except ValueError:
                calls = []
            if calls:
                return None, calls
    return text, []


def message_with_tools(text: str, tools: list[dict] | None, tool_choice: Any, parser: str = "auto"
                       ) -> tuple[dict, bool]:
    """The assistant message of a chat completion whose request declared ``tools``, and
    whether it holds tool calls."""
    name = named_choice(tool_choice)
    if name is not None:  # the constrained output is the arguments object itself
        return {"role": "assistant", "content": None, "tool_calls": [_call(name, text.strip())]}, True
    if tool_choice == "required":
        try:
            calls = _from_obj(json.loads(text), set(_functions(tools)))
        except ValueError:
            calls = []
        if calls:
            return {"role": "assistant", "content": None, "tool_calls": calls}, True
        return {"role": "assistant", "content": text}, False
    content, calls = parse_tool_calls(text, tools, parser)
    if calls:
        return {"role": "assistant", "content": content, "tool_calls": calls}, True
    return {"role": "assistant", "content": text}, False


def tools_prompt(tools: list[dict]) -> str:
    """Plain-text tool description for tokenizers without a chat template."""
    lines = ["You may call these functions. To call one, reply with a JSON object "
             '{"name": <function name>, "arguments": <arguments object>}.']
    for t in tools:
        f = t["function"]
        lines.append(f"- {f['name']}: {f.get('description', '')} parameters: {json.dumps(f.get('parameters', {}))}")
    return "\n".join(lines)
