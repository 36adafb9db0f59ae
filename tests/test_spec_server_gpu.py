"""DSpark speculative decoding through the OpenAI server (GPU, toy V4.1 model).

Concurrent completions are served by :class:`SpecServingEngine` (draft + lossless
verify rounds shared by every admitted request) and must return exactly the
greedy tokens of the same model decoding one token per step; a request asking
for sampling is refused.
"""

import asyncio

import pytest
import torch
from aiohttp.test_utils import TestClient, TestServer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def spec_served():
    from test_dspark_gpu import _greedy, spec_cfg

    from dsv4_flash_deployment_b200.engine.builder import build_model
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.serving.app import ServerState, build_app  # noqa: F401
    from dsv4_flash_deployment_b200.serving.engine_loop import EngineLoop
    from dsv4_flash_deployment_b200.serving.tokenizer import ByteTokenizer
    from dsv4_flash_deployment_b200.spec.dspark import SpecEngine
    from dsv4_flash_deployment_b200.spec.serving import SpecServingEngine

    cfg = spec_cfg()
    w = make_random_weights(cfg, seed=5)
    model = build_model(cfg, "cuda", max_tokens=64, n_slots=4, max_seq_len=160, weights=w)
    eng = SpecServingEngine(SpecEngine(model, w, max_seqs=3), max_seq_len=160)
    loop = EngineLoop(eng).start()
    tok = ByteTokenizer(cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
    st = ServerState(loop, tok, "toy-dspark", 160, {"device": "cuda"})
    ref = build_model(cfg, "cuda", max_tokens=64, n_slots=4, max_seq_len=160, weights=w)
    yield st, eng, (lambda p, n: _greedy(ref, cfg, p, n))
    loop.stop()


def _run(st, coro_fn):
    from dsv4_flash_deployment_b200.serving.app import build_app

    async def main():
        async with TestClient(TestServer(build_app(st))) as c:
            return await coro_fn(c)
    return asyncio.run(main())


def test_spec_server_is_lossless_and_batches(spec_served):
    st, eng, greedy = spec_served
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(10, 1000, (n,), generator=g).tolist() for n in (21, 9, 30, 14)]
    n_new = 17

    async def go(c):
        rs = await asyncio.gather(*(c.post("/v1/completions", json={"prompt": p, "max_tokens": n_new,
                                                                    "ignore_eos": True}) for p in prompts))
        return [await r.json() for r in rs]
    rounds0 = eng.stats["rounds"]
    outs = _run(st, go)
    for p, o in zip(prompts, outs):
        want = greedy(p, n_new)
        assert o["usage"]["completion_tokens"] == n_new
        assert o["choices"][0]["text"] == "".join(st.tok.decode_token(t) for t in want)
        assert o["choices"][0]["finish_reason"] == "length"
    # 4 requests x 17 tokens: rounds are shared (3 rows) and emit >= 1 token each
    assert eng.stats["rounds"] - rounds0 <= 2 * n_new


def test_spec_server_metrics(spec_served):
    st, _, _ = spec_served

    async def go(c):
        return await (await c.get("/metrics")).text()
    text = _run(st, go)
    assert "dsv4_spec_draft_tokens_total" in text and "dsv4_healthy 1" in text


def test_spec_server_refuses_sampling(spec_served):
    st, _, _ = spec_served

    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 3, "temperature": 0.8})
        return r.status, await r.text()
    status, text = _run(st, go)
    assert status == 400 and "greedily" in text
