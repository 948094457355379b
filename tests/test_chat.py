"""Chat glue (host only): ChatML rendering against the reference's corpus
(tests/golden/m12_chatml_corpus.json, expected prompts and rejections made from the upstream
template by the reference's tools/oracle/oracle_chatml.py), the special-token resolver and
tokenizer on the reference's fixture tokenizer (tests/golden/m12_tokenizer), the streaming
detokenizer on split multi-byte characters, the chat turn's control flow on a scripted
engine, and (GPU) a chat turn on the config-0 model against the CPU oracle."""
import io
import json
import os
import shutil

import pytest

from disk_streaming_moe_engine_b200.chat import (ChatMessage, ChatTemplateError, ConfigMismatch, HFTokenizer,
                                                 StreamingDetokenizer, chat_repl, extract_assistant_think,
                                                 render_chatml, resolve_special_tokens, run_chat_turn)

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOKDIR = os.path.join(GOLD, "m12_tokenizer")


def _msgs(case):
    return [ChatMessage(m["role"], m["content"], bool(m.get("has_reasoning_content")), bool(m.get("has_tool_calls")))
            for m in case["messages"]]


def test_render_chatml_matches_reference_corpus():
    corpus = json.load(open(os.path.join(GOLD, "m12_chatml_corpus.json")))
    for case in corpus["valid_cases"]:
        got = render_chatml(_msgs(case), case.get("add_generation_prompt", True))
        assert got == case["expected_prompt"], case["name"]
    for case in corpus["negative_cases"]:
        with pytest.raises(ChatTemplateError) as ei:
            render_chatml(_msgs(case))
        assert case["expected_error"] in str(ei.value), case["name"]


def test_extract_assistant_think():
    assert extract_assistant_think("plain") == ("", "plain")
    assert extract_assistant_think("<think>\nr1\n</think>\n\nanswer") == ("r1", "answer")
    assert extract_assistant_think("a<think>x</think>b<think>y</think>\nc") == ("x", "c")
    assert extract_assistant_think("no open</think>tail") == ("no open", "tail")


def test_streaming_detokenizer_holds_split_characters():
    d = StreamingDetokenizer()
    s = "héllo — 世界 🙂"
    b = s.encode()
    out = "".join(d.feed_bytes(b[i:i + 1]) for i in range(len(b)))
    assert out + d.flush() == s
    d = StreamingDetokenizer()
    assert d.feed_bytes("é".encode()[:1]) == "" and d.feed_bytes("é".encode()[1:]) == "é"
    assert d.feed_bytes(b"\xff") == "�"  # an invalid lead byte passes through


def test_special_tokens_and_tokenizer_fixture(tmp_path):
    r = resolve_special_tokens(TOKDIR, 1024)
    assert (r.im_start_id, r.im_end_id, r.endoftext_id) == (1, 2, 0)
    assert r.is_stop_token(2) and r.is_stop_token(0) and not r.is_stop_token(1)
    tok = HFTokenizer(TOKDIR)
    text = render_chatml([ChatMessage("user", "hello world")])
    ids = tok.encode(text)
    assert ids[0] == r.im_start_id and r.im_end_id in ids and max(ids) < 1024
    assert tok.decode(ids).startswith("<|im_start|>") and tok.encode(text) == ids

    def broken(edit):
        d = tmp_path / f"t{len(list(tmp_path.iterdir()))}"
        shutil.copytree(TOKDIR, d)
        edit(d)
        with pytest.raises(ConfigMismatch) as ei:
            resolve_special_tokens(str(d), 1024)
        return str(ei.value)

    def drop_endoftext(d):
        t = json.load(open(d / "tokenizer.json"))
        t["added_tokens"] = [a for a in t["added_tokens"] if a["content"] != "<|endoftext|>"]
        json.dump(t, open(d / "tokenizer.json", "w"))
    assert "missing required special tokens" in broken(drop_endoftext)

    def bad_eos(d):
        c = json.load(open(d / "tokenizer_config.json"))
        c["eos_token"] = "</s>"
        json.dump(c, open(d / "tokenizer_config.json", "w"))
    assert "eos_token in tokenizer_config.json" in broken(bad_eos)

    def gen_no_eot(d):
        json.dump({"eos_token_id": [2]}, open(d / "generation_config.json", "w"))
    assert "eos_token_id does not contain" in broken(gen_no_eot)

    def id_mismatch(d):
        c = json.load(open(d / "tokenizer_config.json"))
        c["added_tokens_decoder"] = {"5": {"content": "<|im_start|>"}, "2": {"content": "<|im_end|>"},
                                     "0": {"content": "<|endoftext|>"}}
        json.dump(c, open(d / "tokenizer_config.json", "w"))
    assert "id mismatch for <|im_start|>" in broken(id_mismatch)
    with pytest.raises(ConfigMismatch) as ei:
        resolve_special_tokens(TOKDIR, 2)
    assert "TOKEN_INVALID" in str(ei.value)


class _ScriptedEngine:
    """forward / decode_step with scripted greedy ids (records what it was fed)."""

    class cfg:
        vocab_size = 1024

    def __init__(self, prefill_next, steps):
        self.prefill_next, self.steps, self.fed, self.prefills = prefill_next, list(steps), [], []

    def forward(self, tokens, slot=0, want_logits=False):
        self.prefills.append(list(tokens))
        return None, self.prefill_next

    def decode_step(self, tok, slot=0, want_logits=False):
        self.fed.append(tok)
        return self.steps.pop(0), None

    def seq_reset(self, slot):
        pass


def test_chat_turn_control_flow():
    tok = HFTokenizer(TOKDIR)
    res = resolve_special_tokens(TOKDIR, 1024)
    prompt = render_chatml([ChatMessage("user", "hi")])
    a, b = 37, 65  # ordinary vocabulary entries (not stop tokens)
    # reference flow: the last prompt token is fed again; stops at <|im_end|>
    eng = _ScriptedEngine(999, [a, b, res.im_end_id])
    ids, text, fin = run_chat_turn(eng, tok, res, prompt, 10)
    p = tok.encode(prompt)
    assert eng.prefills == [p] and eng.fed == [p[-1], a, b]
    assert ids == [a, b] and fin == "stop" and text == tok.decode([a]) + tok.decode([b])
    # the prefill's own prediction instead; length limit
    eng = _ScriptedEngine(a, [b, b, b])
    ids, _, fin = run_chat_turn(eng, tok, res, prompt, 3, refeed_last=False)
    assert eng.fed == [a, b] and ids == [a, b, b] and fin == "length"
    # the REPL renders the history and streams the reply
    out = io.StringIO()
    hist = chat_repl(_ScriptedEngine(0, [a, res.im_end_id]), TOKDIR, system="sys", stdin=io.StringIO("hi\n/exit\n"),
                     stdout=out)
    assert [m.role for m in hist] == ["system", "user", "assistant"] and out.getvalue() == tok.decode([a]) + "\n"


@pytest.mark.gpu
def test_chat_turn_on_device_matches_oracle(lib, oracle_lib):
    """A chat turn on the config-0 model: the same ids as the CPU oracle driven through the
    same steps (the reference's refeed of the last prompt token included)."""
    import oracle
    from disk_streaming_moe_engine_b200 import Engine, RuntimeConfig, preset, synth
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    tok = HFTokenizer(TOKDIR)
    res = resolve_special_tokens(TOKDIR, cfg.vocab_size)
    prompt = render_chatml([ChatMessage("system", "You are a helpful assistant."), ChatMessage("user", "hello")])
    with Engine(cfg, RuntimeConfig.for_context(256, max_seqs=1)) as eng:
        eng.load_model(m)
        eng.seq_reset(0)
        ids, text, fin = run_chat_turn(eng, tok, res, prompt, 12)
    om = oracle.OracleModel(m)
    st = oracle.OracleState(cfg, 256)
    p = tok.encode(prompt)
    for t in p:
        oracle.decode_step(om, st, int(t))
    want, last = [], p[-1]
    for _ in range(12):
        t, _, _ = oracle.decode_step(om, st, int(last))
        if res.is_stop_token(t):
            break
        want.append(t)
        last = t
    assert ids == want
    assert fin == ("stop" if len(want) < 12 else "length")
