"""Chat prompt rendering.

The reference offers nine built-in formats with model-name auto-detection
(crates/rusteeze-tokenizer/src/chat_template.rs:95-141: Llama, Llama3,
Mistral, ChatML, Zephyr, Vicuna, Alpaca, Phi3, Raw) and silently falls back
to ChatML for a custom template (chat_template.rs:220-482).  Here a Jinja
template from `tokenizer_config.json` (or `--chat-template`) is rendered for
real with jinja2's sandbox when available; the built-in formats are the
fallback and auto-detection follows the same name rules.
"""
from __future__ import annotations

import enum
from typing import Dict, List, Optional


class ChatFormat(str, enum.Enum):
    LLAMA = "llama"
    LLAMA3 = "llama3"
    MISTRAL = "mistral"
    CHATML = "chatml"
    ZEPHYR = "zephyr"
    VICUNA = "vicuna"
    ALPACA = "alpaca"
    PHI3 = "phi3"
    RAW = "raw"

    @classmethod
    def from_model_name(cls, name: str) -> "ChatFormat":
        n = (name or "").lower()
        if "llama-3" in n or "llama3" in n:
            return cls.LLAMA3
        if "llama" in n:
            return cls.LLAMA
        if "mistral" in n or "mixtral" in n:
            return cls.MISTRAL
        if "zephyr" in n:
            return cls.ZEPHYR
        if "vicuna" in n:
            return cls.VICUNA
        if "alpaca" in n:
            return cls.ALPACA
        if "phi-3" in n or "phi3" in n:
            return cls.PHI3
        return cls.CHATML


def _content(m: Dict) -> str:
    c = m.get("content", "")
    if isinstance(c, list):   # multimodal content parts: keep the text parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict) and p.get("type", "text") == "text")
    return c or ""


class ChatTemplate:
    def __init__(self, fmt: ChatFormat = ChatFormat.CHATML, bos: str = "", eos: str = "",
                 jinja: Optional[str] = None):
        self.fmt = ChatFormat(fmt)
        self.bos, self.eos = bos, eos
        self.jinja = jinja

    @classmethod
    def for_model(cls, model_name: str, tokenizer=None, override: Optional[str] = None) -> "ChatTemplate":
        jinja = override or (getattr(tokenizer, "chat_template", None) if tokenizer else None)
        if jinja and jinja in {f.value for f in ChatFormat}:
            return cls(ChatFormat(jinja), getattr(tokenizer, "bos_token", ""), getattr(tokenizer, "eos_token", ""))
        fmt = ChatFormat.from_model_name(model_name)
        bos = getattr(tokenizer, "bos_token", "") if tokenizer else ""
        eos = getattr(tokenizer, "eos_token", "") if tokenizer else ""
        return cls(fmt, bos, eos, jinja)

    def apply(self, messages: List[Dict], add_generation_prompt: bool = True,
              tools: Optional[List[Dict]] = None) -> str:
        """Renders the conversation.  `tools` (OpenAI function definitions) go to a Jinja
        template as its `tools` variable; the built-in formats get them as a system note
        asking for a JSON call, and see tool results and earlier calls as plain turns."""
        if self.jinja:
            try:
                from jinja2.sandbox import ImmutableSandboxedEnvironment
                env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
                env.globals["raise_exception"] = _raise
                return env.from_string(self.jinja).render(
                    messages=[{**m, "content": _content(m)} for m in messages],
                    add_generation_prompt=add_generation_prompt,
                    bos_token=self.bos, eos_token=self.eos, tools=tools)
            except ImportError:
                pass
        msgs = _flatten_tool_turns(messages, tools, self.fmt)
        return getattr(self, f"_{self.fmt.value}")(msgs, add_generation_prompt)

    # ---- built-in formats (public prompt conventions of each model family) ----
    def _llama(self, msgs, gen):
        out, system = [], None
        turns = []
        for m in msgs:
            if m["role"] == "system":
                system = _content(m)
            else:
                turns.append(m)
        first = True
        i = 0
        while i < len(turns):
            m = turns[i]
            if m["role"] == "user":
                u = _content(m)
                if first and system:
                    u = f"<<SYS>>\n{system}\n<</SYS>>\n\n{u}"
                first = False
                out.append(f"{self.bos or '<s>'}[INST] {u.strip()} [/INST]")
                if i + 1 < len(turns) and turns[i + 1]["role"] == "assistant":
                    out.append(f" {_content(turns[i + 1]).strip()} {self.eos or '</s>'}")
                    i += 1
            i += 1
        return "".join(out)

    def _llama3(self, msgs, gen):
        s = "<|begin_of_text|>"
        for m in msgs:
            s += f"<|start_header_id|>{m['role']}<|end_header_id|>\n\n{_content(m).strip()}<|eot_id|>"
        if gen:
            s += "<|start_header_id|>assistant<|end_header_id|>\n\n"
        return s

    def _mistral(self, msgs, gen):
        s = self.bos or "<s>"
        system = "\n\n".join(_content(m) for m in msgs if m["role"] == "system")
        first = True
        for m in msgs:
            if m["role"] == "user":
                u = _content(m)
                if first and system:
                    u = f"{system}\n\n{u}"
                first = False
                s += f"[INST] {u} [/INST]"
            elif m["role"] == "assistant":
                s += f"{_content(m)}{self.eos or '</s>'}"
        return s

    def _chatml(self, msgs, gen):
        s = "".join(f"<|im_start|>{m['role']}\n{_content(m)}<|im_end|>\n" for m in msgs)
        return s + ("<|im_start|>assistant\n" if gen else "")

    def _zephyr(self, msgs, gen):
        eos = self.eos or "</s>"
        s = "".join(f"<|{m['role']}|>\n{_content(m)}{eos}\n" for m in msgs)
        return s + ("<|assistant|>\n" if gen else "")

    def _vicuna(self, msgs, gen):
        s = ""
        for m in msgs:
            if m["role"] == "system":
                s += _content(m) + "\n\n"
            elif m["role"] == "user":
                s += f"USER: {_content(m)}\n"
            else:
                s += f"ASSISTANT: {_content(m)}{self.eos or '</s>'}\n"
        return s + ("ASSISTANT:" if gen else "")

    def _alpaca(self, msgs, gen):
        s = ""
        for m in msgs:
            if m["role"] == "system":
                s += _content(m) + "\n\n"
            elif m["role"] == "user":
                s += f"### Instruction:\n{_content(m)}\n\n"
            else:
                s += f"### Response:\n{_content(m)}\n\n"
        return s + ("### Response:\n" if gen else "")

    def _phi3(self, msgs, gen):
        s = "".join(f"<|{m['role']}|>\n{_content(m)}<|end|>\n" for m in msgs)
        return s + ("<|assistant|>\n" if gen else "")

    def _raw(self, msgs, gen):
        return "\n".join(_content(m) for m in msgs)


def _raise(msg):
    raise ValueError(msg)


_ROLE_FORMATS = ("chatml", "llama3", "zephyr", "phi3")


def _flatten_tool_turns(messages: List[Dict], tools: Optional[List[Dict]], fmt) -> List[Dict]:
    """Tool definitions, calls and results as ordinary turns for the built-in formats:
    the definitions as a system note, an assistant's calls as JSON in its content, a tool
    result under the `tool` role where the format has named roles (else as a user turn)."""
    import json
    out: List[Dict] = []
    if tools:
        fns = [t.get("function", t) for t in tools]
        note = ("You can call these functions. To call one, answer with only a JSON object "
                '{"name": <function name>, "arguments": <arguments object>}.\n' + json.dumps(fns))
        out.append({"role": "system", "content": note})
    for m in messages:
        m = dict(m)
        calls = m.get("tool_calls")
        if m.get("role") == "assistant" and calls:
            parts = [_content(m)] if _content(m) else []
            for c in calls:
                f = c.get("function", {})
                args = f.get("arguments", "{}")
                parts.append(json.dumps({"name": f.get("name"),
                                         "arguments": json.loads(args) if isinstance(args, str) else args}))
            m["content"] = "\n".join(parts)
        if m.get("role") == "tool" and getattr(fmt, "value", fmt) not in _ROLE_FORMATS:
            m["role"] = "user"
            m["content"] = f"Tool result: {_content(m)}"
        out.append(m)
    return out
