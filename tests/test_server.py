"""OpenAI-compatible server on the CPU oracle engine (toy V4 model).

Checks the API surface the reference's server and sweep client use: health,
models, tokenize, completions (plain / streamed / token-id prompts / stop
strings / length errors), chat completions, metrics, and that concurrent
requests share engine steps and get the oracle's greedy tokens.
"""

import asyncio
import json

import pytest
import torch
from aiohttp.test_utils import TestClient, TestServer

from dsv4_flash_deployment_b200.engine.config import EngineConfig
from dsv4_flash_deployment_b200.ref.model import RefModel
from dsv4_flash_deployment_b200.serving.app import ServerState, build_app
from dsv4_flash_deployment_b200.serving.engine_loop import EngineLoop
from dsv4_flash_deployment_b200.serving.launch import build_local_engine
from dsv4_flash_deployment_b200.serving.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def served():
    ec = EngineConfig(device="cpu", model="toy-v4", max_seqs=4, max_batched_tokens=48, chunk_size=16,
                      max_model_len=160, served_model_name="toy")
    eng = build_local_engine(ec)
    loop = EngineLoop(eng).start()
    tok = ByteTokenizer(eng.cfg.vocab_size, eng.cfg.bos_token_id, eng.cfg.eos_token_id)
    st = ServerState(loop, tok, "toy", ec.max_model_len, {"device": "cpu"})
    yield st, eng
    loop.stop()


def _run(st, coro_fn):
    async def main():
        async with TestClient(TestServer(build_app(st))) as c:
            return await coro_fn(c)
    return asyncio.run(main())


def _greedy(eng, ids, n):
    ref = RefModel(eng.cfg, eng.model.ref.w, max_seq_len=256)
    out, _ = ref.generate(torch.tensor([ids]), n)
    return out[0].tolist()


def test_health_models_tokenize(served):
    st, _ = served

    async def go(c):
        h = await (await c.get("/health")).json()
        m = await (await c.get("/v1/models")).json()
        t = await (await c.post("/tokenize", json={"model": "toy", "prompt": "hello"})).json()
        d = await (await c.post("/detokenize", json={"tokens": t["tokens"]})).json()
        return h, m, t, d
    h, m, t, d = _run(st, go)
    assert h["status"] == "ok" and h["model"] == "toy"
    assert m["data"][0]["id"] == "toy"
    assert t["count"] == 6 and t["max_model_len"] == 160   # bos + 5 bytes
    assert d["prompt"] == "hello"


def test_completion_matches_oracle_and_streams(served):
    st, eng = served
    ids = [0] + [20 + (7 * i) % 200 for i in range(40)]

    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 6, "ignore_eos": True})
        body = await r.json()
        r2 = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 6, "ignore_eos": True,
                                                   "stream": True})
        chunks, done = [], False
        async for raw in r2.content:
            line = raw.decode().strip()
            if not line.startswith("data: "):
                continue
            if line[6:] == "[DONE]":
                done = True
                break
            chunks.append(json.loads(line[6:]))
        return body, chunks, done
    body, chunks, done = _run(st, go)
    want = _greedy(eng, ids, 6)
    tok = st.tok
    assert body["usage"]["completion_tokens"] == 6
    assert body["choices"][0]["text"] == "".join(tok.decode_token(t) for t in want)
    assert body["choices"][0]["finish_reason"] == "length"
    texts = [c["choices"][0]["text"] for c in chunks if c["choices"][0]["text"]]
    assert done and len(texts) == 6 and "".join(texts) == body["choices"][0]["text"]
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"


def test_concurrent_requests_share_steps(served):
    st, eng = served
    prompts = [[0] + [30 + (i * 13 + j) % 150 for j in range(20 + 9 * i)] for i in range(3)]
    steps0 = eng.stats["steps"]

    async def go(c):
        rs = await asyncio.gather(*(c.post("/v1/completions", json={"prompt": p, "max_tokens": 5,
                                                                    "ignore_eos": True}) for p in prompts))
        return [await r.json() for r in rs]
    outs = _run(st, go)
    for p, o in zip(prompts, outs):
        want = _greedy(eng, p, 5)
        assert o["choices"][0]["text"] == "".join(st.tok.decode_token(t) for t in want)
    # 3 requests x (prefill + 5 tokens) in far fewer steps than serially
    assert eng.stats["steps"] - steps0 < 3 * 9


def test_chat_stop_and_errors(served):
    st, eng = served

    async def go(c):
        chat = await (await c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "ignore_eos": True})).json()
        too_long = await c.post("/v1/completions", json={"prompt": "x" * 150, "max_tokens": 20})
        bad = await c.post("/v1/completions", data=b"{not json")
        full = await (await c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 8,
                                                            "ignore_eos": True})).json()
        text = full["choices"][0]["text"]
        stop = text[len(text) // 2: len(text) // 2 + 2] if len(text) > 3 else None
        stopped = None
        if stop:
            stopped = await (await c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 8,
                                                                   "ignore_eos": True, "stop": [stop]})).json()
        metrics = await (await c.get("/metrics")).text()
        return chat, too_long.status, bad.status, text, stop, stopped, metrics
    chat, too_long, bad, text, stop, stopped, metrics = _run(st, go)
    assert chat["object"] == "chat.completion" and chat["usage"]["completion_tokens"] == 3
    assert chat["choices"][0]["message"]["role"] == "assistant"
    assert too_long == 400 and bad == 400
    if stop:
        assert stopped["choices"][0]["finish_reason"] == "stop"
        assert stopped["choices"][0]["text"] == text[:text.find(stop)]
    assert "dsv4_generation_tokens_total" in metrics and "dsv4_healthy 1" in metrics


def test_sweep_client_rows(served, tmp_path):
    from dsv4_flash_deployment_b200.bench.sweep import sweep

    st, _ = served
    out = tmp_path / "rows.json"

    async def go(c):
        base = str(c.make_url("")).rstrip("/")
        shape = {"isl": 24, "osl": 4, "min_reqs": 2, "label": "tiny"}
        rows = await sweep(base, "toy", shape, "tiny", [1, 3], str(out), n_gpus=1, vocab=1024, max_model_len=160)
        words = await sweep(base, "toy", shape, "tiny", [2], None, n_gpus=1, prompt_mode="words")
        return rows, words
    rows, words = _run(st, go)
    saved = json.loads(out.read_text())
    assert [r["concurrency"] for r in saved] == [1, 3]
    for r in rows + words:
        assert r["failed"] == 0 and r["success_rate_pct"] == 100.0
        assert r["output_tokens"] == 4 * r["requests_issued"]
        assert r["ttft_mean_ms"] > 0 and r["tpot_mean_ms"] > 0
        for k in ("output_throughput_tok_s", "output_tok_s_per_chip", "requests_per_s", "ttft_p50_ms",
                  "ttft_p90_ms", "wall_time_s", "isl_min", "isl_max", "osl", "started_at", "first_error"):
            assert k in r
    assert words[0]["isl_max"] <= 24 and words[0]["n_words"] > 0


def test_client_smoke_and_determinism(served):
    from dsv4_flash_deployment_b200.bench.client_checks import determinism, smoke

    st, _ = served

    async def go(c):
        base = str(c.make_url("")).rstrip("/")
        return await smoke(base, "toy"), await determinism(base, "toy", n=6, max_tokens=3, concurrency=4, max_words=12)
    s, d = _run(st, go)
    assert s["ok"], s
    assert d["ok"] and d["n"] == 6, d


def test_eval_client_scores_and_resumes(served, tmp_path):
    from dsv4_flash_deployment_b200.bench import evals

    st, _ = served
    mc = [{"question": f"q{i}", "choices": ["w", "x", "y", "z"], "answer": "C"} for i in range(4)]
    math = [{"question": f"{i}+1", "answer": f"work #### {i + 1}"} for i in range(3)]
    part = str(tmp_path / "mc.partial.jsonl")

    async def go(c):
        base = str(c.make_url("")).rstrip("/")
        a = await evals.run_eval("mc", base, "toy", mc, 4, 0.0, 2, part, seed=1, template="{question} {options}")
        b = await evals.run_eval("mc", base, "toy", mc, 4, 0.0, 2, part, seed=1, template="{question} {options}")
        m = await evals.run_eval("math", base, "toy", math, 4, 0.0, 3, None, template="{question}=")
        return a, b, m
    a, b, m = _run(st, go)
    assert a["n"] == 4 and a["errors"] == 0 and a["resumed"] == 0 and a["verdict"]["complete"]
    assert b["n"] == 4 and b["resumed"] == 4           # every item came from the partial file
    assert sum(1 for _ in open(part)) == 4
    assert m["n"] == 3 and m["errors"] == 0


def test_eval_parsing_and_shuffle():
    from dsv4_flash_deployment_b200.bench import evals

    item = {"question": "Q", "choices": ["right", "a", "b", "c"], "answer": 0}
    p1, t1 = evals.mc_prompt(item, 5, 0)
    p2, t2 = evals.mc_prompt(item, 5, 0)
    assert (p1, t1) == (p2, t2)                        # seeded per (seed, item)
    assert f"{t1}) right" in p1
    assert evals.extract_letter("so...\nAnswer: (b)\n") == "B"
    assert evals.extract_letter("Answer: A then Answer: **D**") == "D"
    assert evals.extract_letter("no letter") is None
    assert evals.math_target({"answer": "steps #### 1,234"}) == 1234.0
    assert evals._number("the result is -3.5.") == -3.5


def test_temperature_sampling_and_refusals(served):
    st, eng = served
    ids = [0] + [30 + (5 * i) % 200 for i in range(30)]
    want = _greedy(eng, ids, 8)

    async def go(c):
        g = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 8, "ignore_eos": True,
                                                          "temperature": 0})).json()
        hot = []
        for _ in range(3):
            r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 8, "ignore_eos": True,
                                                      "temperature": 5.0, "top_p": 1.0})
            hot.append(await r.json())
        bad = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 2, "top_p": 1.5})
        neg = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 2, "temperature": -1})
        for extra in ({"n": 0}, {"best_of": 3}, {"logprobs": 21}, {"top_p": 0}, {"top_k": "x"}, {"n": 65}):
            r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 2, **extra})
            assert r.status == 400, extra
        ok = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 2, "n": 1, "logprobs": None})
        assert ok.status == 200
        return g, hot, bad.status, neg.status
    g, hot, bad, neg = _run(st, go)
    tok = st.tok
    assert g["choices"][0]["text"] == "".join(tok.decode_token(t) for t in want)
    texts = [h["choices"][0]["text"] for h in hot]
    assert all(h["usage"]["completion_tokens"] == 8 for h in hot)
    # a near-flat random-init distribution at T=5: three samples of 8 tokens are not all the greedy text
    assert any(t != g["choices"][0]["text"] for t in texts)
    assert bad == 400 and neg == 400


def test_logprobs_and_nucleus_sampling(served):
    """Completions and chat return per-token log-probabilities in the OpenAI
    layouts; the greedy token's log-probability is its top alternative's and
    equals log_softmax of the oracle logits; top-k 1 at any temperature decodes
    greedily, and top-p / top-k samples stay within their sets."""
    st, eng = served
    ids = [0] + [40 + (3 * i) % 150 for i in range(25)]
    want = _greedy(eng, ids, 5)

    async def go(c):
        comp = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 5, "ignore_eos": True,
                                                             "logprobs": 3})).json()
        chat = await (await c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hi"}], "max_tokens": 4, "ignore_eos": True,
            "logprobs": True, "top_logprobs": 2})).json()
        k1 = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 5, "ignore_eos": True,
                                                           "temperature": 3.0, "top_k": 1})).json()
        streamed = []
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 3, "ignore_eos": True,
                                                  "logprobs": 1, "stream": True})
        async for raw in r.content:
            line = raw.decode().strip()
            if line.startswith("data: {"):
                streamed.append(json.loads(line[6:]))
        return comp, chat, k1, streamed
    comp, chat, k1, streamed = _run(st, go)
    tok = st.tok
    lp = comp["choices"][0]["logprobs"]
    assert lp["tokens"] == [tok.decode_token(t) for t in want]
    assert len(lp["token_logprobs"]) == 5 and all(len(d) <= 3 for d in lp["top_logprobs"])
    assert lp["text_offset"][0] == 0
    for piece, v, tops in zip(lp["tokens"], lp["token_logprobs"], lp["top_logprobs"]):
        assert v <= 0 and abs(max(tops.values()) - v) < 1e-5 and tops.get(piece) is not None
    # the first token's value against the oracle's own logits
    ref = RefModel(eng.cfg, eng.model.ref.w, max_seq_len=256)
    st0 = ref.new_state(1)
    for t in ids:
        logits, _ = ref.step(torch.tensor([t]), st0)
    lsm = torch.log_softmax(logits[0].float()[: eng.cfg.vocab_size], -1)
    assert abs(lsm[want[0]].item() - lp["token_logprobs"][0]) < 1e-4
    c = chat["choices"][0]["logprobs"]["content"]
    assert len(c) == 4 and all(len(e["top_logprobs"]) == 2 and e["logprob"] <= 0 for e in c)
    assert all(e["bytes"] == list(e["token"].encode()) for e in c)
    assert k1["choices"][0]["text"] == "".join(tok.decode_token(t) for t in want)
    pieces = [ch["choices"][0]["logprobs"] for ch in streamed if ch["choices"][0]["text"]]
    assert len(pieces) == 3 and all(len(p["tokens"]) == 1 for p in pieces)


def test_n_choices_and_batched_prompts(served):
    """A list of prompts times n choices: greedy choices equal the oracle per
    prompt with index = prompt * n + j; seeded sampled choices repeat on a second
    request; a streamed request tags every chunk with its choice index."""
    st, eng = served
    p1 = [0] + [50 + (3 * i) % 120 for i in range(14)]
    p2 = [0] + [60 + (7 * i) % 110 for i in range(9)]
    w1, w2 = _greedy(eng, p1, 4), _greedy(eng, p2, 4)

    async def go(c):
        batch = await (await c.post("/v1/completions", json={"prompt": [p1, p2], "n": 2, "max_tokens": 4,
                                                              "ignore_eos": True})).json()
        body = {"messages": [{"role": "user", "content": "pick"}], "n": 3, "max_tokens": 5, "ignore_eos": True,
                "temperature": 3.0, "seed": 11}
        s1 = await (await c.post("/v1/chat/completions", json=body)).json()
        s2 = await (await c.post("/v1/chat/completions", json=body)).json()
        r = await c.post("/v1/completions", json={"prompt": p1, "n": 2, "max_tokens": 4, "ignore_eos": True,
                                                  "stream": True})
        parts = {}
        async for raw in r.content:
            line = raw.decode().strip()
            if line.startswith("data: {"):
                ch = json.loads(line[6:])["choices"][0]
                parts.setdefault(ch["index"], []).append(ch["text"])
        return batch, s1, s2, parts
    batch, s1, s2, parts = _run(st, go)
    tok = st.tok
    t1, t2 = ("".join(tok.decode_token(t) for t in w) for w in (w1, w2))
    ch = sorted(batch["choices"], key=lambda c: c["index"])
    assert [c["index"] for c in ch] == [0, 1, 2, 3]
    assert [c["text"] for c in ch] == [t1, t1, t2, t2]
    assert batch["usage"]["completion_tokens"] == 16 and batch["usage"]["prompt_tokens"] == len(p1) + len(p2)
    a = {c["index"]: c["message"]["content"] for c in s1["choices"]}
    b = {c["index"]: c["message"]["content"] for c in s2["choices"]}
    assert a == b and sorted(a) == [0, 1, 2]
    assert len(set(a.values())) > 1        # choices draw with seeds 11, 12, 13
    assert {i: "".join(v) for i, v in parts.items()} == {0: t1, 1: t1}


def test_streamed_chat_chunks_parse_and_match_the_full_answer(served):
    st, _ = served
    body = {"messages": [{"role": "user", "content": "stream me"}], "max_tokens": 6, "ignore_eos": True}

    async def go(c):
        full = await (await c.post("/v1/chat/completions", json=body)).json()
        r = await c.post("/v1/chat/completions", json={**body, "stream": True})
        chunks = []
        async for raw in r.content:
            line = raw.decode().strip()
            if line.startswith("data: {"):
                chunks.append(json.loads(line[6:]))
        return full, chunks
    full, chunks = _run(st, go)
    deltas = [c["choices"][0]["delta"] for c in chunks]
    assert deltas[0].get("role") == "assistant"
    assert all(c["object"] == "chat.completion.chunk" and c["id"] == chunks[0]["id"] for c in chunks)
    assert "".join(d.get("content", "") for d in deltas) == full["choices"][0]["message"]["content"]
    assert chunks[-1]["choices"][0]["finish_reason"] == "length" and "usage" in chunks[-1]


def test_api_key_guards_the_api_but_not_health(served):
    st, _ = served

    async def go(c):
        st.api_key = "s3cret"
        try:
            no = await c.post("/v1/completions", json={"prompt": [0, 5], "max_tokens": 1})
            bad = await c.get("/v1/models", headers={"Authorization": "Bearer nope"})
            ok = await c.get("/v1/models", headers={"Authorization": "Bearer s3cret"})
            health = await c.get("/health")
            return no.status, bad.status, ok.status, health.status
        finally:
            st.api_key = None
    assert _run(st, go) == (401, 401, 200, 200)
    from dsv4_flash_deployment_b200.engine.config import EngineConfig
    assert EngineConfig(api_key="k").to_dict()["api_key"] == "(set)"


def test_stream_usage_chunk_and_echo(served):
    st, eng = served
    ids = [0] + [33 + (5 * i) % 100 for i in range(8)]

    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 3, "ignore_eos": True, "stream": True,
                                                  "stream_options": {"include_usage": True}})
        chunks = []
        async for raw in r.content:
            line = raw.decode().strip()
            if line.startswith("data: {"):
                chunks.append(json.loads(line[6:]))
        e = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 3, "ignore_eos": True,
                                                          "echo": True})).json()
        plain = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 3,
                                                              "ignore_eos": True})).json()
        return chunks, e, plain
    chunks, e, plain = _run(st, go)
    assert chunks[-1]["choices"] == [] and chunks[-1]["usage"]["completion_tokens"] == 3
    assert all("usage" not in ch for ch in chunks[:-1])
    assert e["choices"][0]["text"] == st.tok.decode(ids) + plain["choices"][0]["text"]


def test_incremental_decoder_holds_back_split_characters():
    from dsv4_flash_deployment_b200.serving.tokenizer import ByteTokenizer, IncrementalDecoder

    tok = ByteTokenizer(1024)
    text = "añ€😀 ok"
    ids = tok.encode(text, add_bos=False)
    dec = IncrementalDecoder(tok.decode)
    pieces = [dec.push(t) for t in ids]
    assert "".join(pieces) + dec.flush() == text
    assert all("�" not in p for p in pieces)
    assert pieces.count("") == len(ids) - len(text)      # one empty piece per continuation byte
    # a character cut off at the end comes out of flush as U+FFFD
    dec = IncrementalDecoder(tok.decode)
    got = [dec.push(t) for t in tok.encode("x€", add_bos=False)[:-1]]
    assert "".join(got) == "x" and dec.flush() == "�"


def test_server_streams_whole_characters_with_an_incremental_tokenizer(served):
    """A tokenizer whose tokens are bytes (as byte-level BPE ones are): the streamed
    pieces never split a character and add up to the text of all generated ids."""
    from dsv4_flash_deployment_b200.serving.tokenizer import ByteTokenizer, IncrementalDecoder

    st, eng = served

    class ByteLevel(ByteTokenizer):
        def stream_decoder(self):
            return IncrementalDecoder(self.decode)

    old = st.tok
    st.tok = ByteLevel(old.vocab_size, old.bos_token_id, old.eos_token_id)
    ids = [0] + [40 + (9 * i) % 150 for i in range(10)]

    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 12, "ignore_eos": True,
                                                  "stream": True})
        pieces = []
        async for raw in r.content:
            line = raw.decode().strip()
            if line.startswith("data: {"):
                ch = json.loads(line[6:])["choices"]
                if ch and ch[0]["text"]:
                    pieces.append(ch[0]["text"])
        full = await (await c.post("/v1/completions", json={"prompt": ids, "max_tokens": 12,
                                                             "ignore_eos": True})).json()
        return pieces, full
    try:
        pieces, full = _run(st, go)
    finally:
        st.tok = old
    want = st.tok.decode(_greedy(eng, ids, 12))
    assert "".join(pieces) == full["choices"][0]["text"] == want
