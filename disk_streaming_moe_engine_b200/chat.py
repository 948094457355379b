"""Chat glue over the decode step: ChatML rendering, special tokens, tokenizer, streaming
detokenizer and the chat turn / REPL (host-only; the model runs in libdismoen_cuda.so).

Restates the reference's text-only Qwen3.6 chat subset:
  render_chatml / extract_assistant_think / extract_last_query_index
                           src/tokenizer/chatml.mojo:64-232 (rejections with its messages)
  StreamingDetokenizer     src/tokenizer/detokenizer.mojo:17-131
  resolve_special_tokens   src/tokenizer/special_tokens.mojo:134-262 (CONFIG_MISMATCH /
                           TOKEN_INVALID checks)
  HFTokenizer              tools/tokenizer_cli.py (the reference encodes and decodes through
                           the `tokenizers` library: encode(text).ids,
                           decode(ids, skip_special_tokens=False))
  run_chat_turn            src/cli/cmd_chat.mojo:199-339: encode, prefill, greedy decode
                           until a stop token or max_tokens, text streamed per token
"""
from __future__ import annotations

import json
import os
import sys
from dataclasses import dataclass

import numpy as np


class ChatTemplateError(ValueError):
    """An input outside the rendered subset ("400 Bad Request: unsupported: ..." or 422)."""


class ConfigMismatch(ValueError):
    """Special-token metadata that fails the resolver's checks (CONFIG_MISMATCH / TOKEN_INVALID)."""


@dataclass
class ChatMessage:
    role: str
    content: str
    has_reasoning_content: bool = False
    has_tool_calls: bool = False


def extract_assistant_think(raw: str) -> tuple[str, str]:
    """(reasoning, content) of an assistant message, as the upstream template splits it."""
    if "</think>" not in raw:
        return "", raw.strip()
    before = raw[:raw.find("</think>")].rstrip("\n")
    reasoning = before.split("<think>")[-1].lstrip("\n")
    after = raw.split("</think>")[-1].lstrip("\n")
    return reasoning.strip(), after.strip()


def extract_last_query_index(messages: list[ChatMessage]) -> int:
    for i in range(len(messages) - 1, -1, -1):
        if messages[i].role == "user":
            t = messages[i].content.strip()
            if not (t.startswith("<tool_response>") and t.endswith("</tool_response>")):
                return i
    return -1


def render_chatml(messages: list[ChatMessage], add_generation_prompt: bool = True) -> str:
    if not messages:
        raise ChatTemplateError("400 Bad Request: unsupported: empty_messages")
    for m in messages:
        if m.has_reasoning_content:
            raise ChatTemplateError("422 Unprocessable Entity: unsupported: field=reasoning_content")
        if m.has_tool_calls:
            raise ChatTemplateError("422 Unprocessable Entity: unsupported: field=tool_calls")
        if m.role not in ("system", "user", "assistant"):
            raise ChatTemplateError("400 Bad Request: unsupported: role=" + m.role)
    n_sys = 0
    for i, m in enumerate(messages):
        if m.role == "system":
            n_sys += 1
            if i != 0:
                raise ChatTemplateError("400 Bad Request: unsupported: " +
                                        ("duplicate_system" if n_sys > 1 else "system_not_first"))
    last = extract_last_query_index(messages)
    if last == -1:
        raise ChatTemplateError("400 Bad Request: unsupported: no_user_query")
    out = []
    if messages[0].role == "system":
        out.append("<|im_start|>system\n" + messages[0].content.strip() + "<|im_end|>\n")
    for i, m in enumerate(messages):
        if m.role == "user":
            out.append("<|im_start|>user\n" + m.content.strip() + "<|im_end|>\n")
        elif m.role == "assistant":
            reasoning, content = extract_assistant_think(m.content)
            if i > last:  # trailing assistant turn: its reasoning stays, wrapped
                out.append("<|im_start|>assistant\n<think>\n" + reasoning + "\n</think>\n\n" + content +
                           "<|im_end|>\n")
            else:
                out.append("<|im_start|>assistant\n" + content + "<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n<think>\n")
    return "".join(out)


class StreamingDetokenizer:
    """Buffers bytes and releases only complete UTF-8 sequences; invalid lead or
    continuation bytes pass through one at a time."""

    def __init__(self):
        self.buffer = bytearray()

    def feed_bytes(self, data: bytes) -> str:
        self.buffer.extend(data)
        return self._consume()

    def feed_string(self, text: str) -> str:
        return self.feed_bytes(text.encode("utf-8", errors="surrogatepass"))

    def _consume(self) -> str:
        b = self.buffer
        i = end = 0
        n = len(b)
        while i < n:
            c = b[i]
            need = 1 if c < 0x80 else 2 if (c & 0xE0) == 0xC0 else 3 if (c & 0xF0) == 0xE0 else \
                4 if (c & 0xF8) == 0xF0 else 0
            if need <= 1:  # ASCII or an invalid lead byte
                i += 1
                end = i
                continue
            if i + need - 1 >= n:
                break  # incomplete at the end: keep it
            if all((b[i + k] & 0xC0) == 0x80 for k in range(1, need)):
                i += need
            else:
                i += 1
            end = i
        out = bytes(b[:end])
        del b[:end]
        return out.decode("utf-8", errors="replace")

    def flush(self) -> str:
        out = bytes(self.buffer)
        self.buffer.clear()
        return out.decode("utf-8", errors="replace")


@dataclass
class SpecialTokenResolver:
    im_start_id: int
    im_end_id: int
    endoftext_id: int
    eos_token_ids: list[int]
    eos_token_str: str

    def is_stop_token(self, token_id: int) -> bool:
        return token_id in self.eos_token_ids


_SPECIAL = ("<|im_start|>", "<|im_end|>", "<|endoftext|>")


def _load_json(path: str, what: str):
    try:
        with open(path, "r", encoding="utf-8") as f:
            return json.load(f)
    except Exception as e:
        raise ConfigMismatch(f"CONFIG_MISMATCH: cannot open {what}: {e}") from None


def resolve_special_tokens(model_dir: str, vocab_size: int = 248320) -> SpecialTokenResolver:
    tok = _load_json(os.path.join(model_dir, "tokenizer.json"), "tokenizer.json")
    ids = {}
    for t in tok.get("added_tokens", []):
        if t.get("content") in _SPECIAL:
            ids[t["content"]] = int(t["id"])
    if len(ids) != 3:
        raise ConfigMismatch("CONFIG_MISMATCH: tokenizer.json missing required special tokens "
                             "(<|im_start|>, <|im_end|>, <|endoftext|>)")
    cfg = _load_json(os.path.join(model_dir, "tokenizer_config.json"), "tokenizer_config.json")
    dec = {v.get("content"): int(k) for k, v in cfg.get("added_tokens_decoder", {}).items()}
    for s in _SPECIAL:
        if s in dec and dec[s] != ids[s]:
            raise ConfigMismatch(f"CONFIG_MISMATCH: id mismatch for {s} between tokenizer.json and "
                                 "tokenizer_config.json")
    if not all(s in dec for s in _SPECIAL):
        raise ConfigMismatch("CONFIG_MISMATCH: tokenizer_config.json added_tokens_decoder is missing required "
                             "special tokens")
    eos = cfg.get("eos_token", "")
    if isinstance(eos, dict):
        eos = eos.get("content", "")
    if eos not in _SPECIAL:
        raise ConfigMismatch(f"CONFIG_MISMATCH: eos_token in tokenizer_config.json ('{eos}') does not refer to a "
                             "valid special token (<|im_start|>, <|im_end|>, <|endoftext|>)")
    gen = _load_json(os.path.join(model_dir, "generation_config.json"), "generation_config.json")
    eos_ids = gen.get("eos_token_id", [])
    eos_ids = [int(x) for x in (eos_ids if isinstance(eos_ids, list) else [eos_ids])]
    if ids["<|im_end|>"] not in eos_ids or ids["<|endoftext|>"] not in eos_ids:
        raise ConfigMismatch("CONFIG_MISMATCH: generation_config.json eos_token_id does not contain required "
                             "stop tokens {<|im_end|>, <|endoftext|>}")
    vs = vocab_size
    try:
        mc = json.load(open(os.path.join(model_dir, "config.json"), encoding="utf-8"))
        if int(mc.get("vocab_size", 0)) > 0:
            vs = int(mc["vocab_size"])
    except Exception:
        pass
    for s in _SPECIAL:
        if not 0 <= ids[s] < vs:
            raise ConfigMismatch(f"TOKEN_INVALID: {s} id {ids[s]} outside vocab_size range [0, {vs})")
    return SpecialTokenResolver(ids["<|im_start|>"], ids["<|im_end|>"], ids["<|endoftext|>"], eos_ids, eos)


class HFTokenizer:
    """The model's tokenizer.json through the `tokenizers` library (no fallback)."""

    def __init__(self, model_dir: str):
        path = os.path.join(model_dir, "tokenizer.json")
        if not os.path.exists(path):
            raise FileNotFoundError(f"TOKENIZER_NOT_FOUND: no tokenizer.json in model dir: {model_dir!r}")
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text).ids

    def decode(self, ids) -> str:
        return self.tok.decode([int(i) for i in ids], skip_special_tokens=False)


def run_chat_turn(engine, tokenizer, resolver: SpecialTokenResolver, prompt_rendered: str, max_tokens: int,
                  slot: int = 0, on_text=None, refeed_last: bool = True):
    """One turn: encode, prefill the prompt into `slot` (after whatever the slot holds),
    greedy-decode until a stop token or max_tokens; returns (generated ids, text,
    finish_reason "stop" | "length").  The reference feeds the last prompt token once
    more before the first generated one (cmd_chat.mojo:272-285: the prefill's own
    prediction is not used); refeed_last=False takes the prefill's prediction instead."""
    prompt = tokenizer.encode(prompt_rendered)
    if not prompt:
        raise ValueError("prompt encodes to 0 tokens")
    _, nxt = engine.forward(np.asarray(prompt, np.int32), slot=slot, want_logits=False)
    detok = StreamingDetokenizer()
    generated, text, finish = [], [], "length"
    last = prompt[-1]
    for step in range(max_tokens):
        if refeed_last or step > 0:
            tok, _ = engine.decode_step(int(last), slot=slot, want_logits=False)
        else:
            tok = nxt
        if resolver.is_stop_token(tok):
            finish = "stop"
            break
        generated.append(tok)
        last = tok
        piece = detok.feed_string(tokenizer.decode([tok]))
        text.append(piece)
        if piece and on_text:
            on_text(piece)
    tail = detok.flush()
    if tail:
        text.append(tail)
        if on_text:
            on_text(tail)
    return generated, "".join(text), finish


def chat_repl(engine, model_dir: str, system: str = "", max_tokens: int = 512, slot: int = 0,
              stdin=None, stdout=None):
    """Line-oriented chat (cmd_chat.mojo): each user line joins the history, the whole
    rendered conversation is prefilled into a fresh slot (the rendering drops earlier
    turns' reasoning, so the slot's old state is not a prefix of it) and the reply streams
    to stdout.  "/exit" ends, "/reset" clears the history."""
    stdin = stdin or sys.stdin
    stdout = stdout or sys.stdout
    tok = HFTokenizer(model_dir)
    res = resolve_special_tokens(model_dir, engine.cfg.vocab_size)
    history = [ChatMessage("system", system)] if system else []
    for line in stdin:
        line = line.rstrip("\n")
        if line == "/exit":
            break
        if line == "/reset":
            history = [ChatMessage("system", system)] if system else []
            continue
        history.append(ChatMessage("user", line))
        engine.seq_reset(slot)
        _, text, _ = run_chat_turn(engine, tok, res, render_chatml(history), max_tokens, slot,
                                   on_text=lambda s: (stdout.write(s), stdout.flush()))
        stdout.write("\n")
        history.append(ChatMessage("assistant", text))
    return history
