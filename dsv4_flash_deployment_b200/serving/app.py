"""OpenAI-compatible HTTP server.

Endpoints (the union of the reference's ``tpu-v7x/deepseek_v41/server.py``
and what its sweep client asks of vLLM, ``kernel-optimizations-recipe/
scripts/benchmark_sweep.py:70-125``):

  GET  /health                 status, model, device, totals (503 when the engine is unhealthy)
  GET  /v1/models              the served model id
  GET  /metrics                Prometheus text: requests, tokens, step time, batch, TTFT, slots
  POST /tokenize               {"prompt"} or {"messages"} -> {"count", "tokens", "max_model_len"}
  POST /detokenize             {"tokens"} -> {"prompt"}
  POST /v1/completions         prompt (text | ids | [text]), max_tokens, stream, ignore_eos, stop
  POST /v1/chat/completions    messages, max_tokens / max_completion_tokens, stream, stop

Decoding: ``temperature`` 0 (the default when the field is absent, and what
every reference benchmark sends) is greedy; ``temperature`` > 0 samples
softmax(logits / T) on the device by the Gumbel-max rule, restricted by
``top_k`` (> 0) and ``top_p`` (< 1) when given; ``seed`` makes the samples a
function of (seed, position) only, so a seeded request repeats its output.  ``logprobs`` (completions: the
number of alternatives, 0-20; chat: ``logprobs: true`` with ``top_logprobs``
0-20) returns each generated token's log-probability under the raw logits and
its most likely alternatives, in the OpenAI response layouts.  ``n`` /
``best_of`` > 1 are refused with 400, and so is any request the engine cannot
serve (top-k / top-p / logprobs on the tensor-parallel head, logprobs or
temperature under speculative decoding).
Streaming sends one SSE event per generated token and ends with
``data: [DONE]``; a client that disconnects cancels its request.

Run: ``python -m dsv4_flash_deployment_b200.serving --config v4-flash --port 8000``.
"""

from __future__ import annotations

import asyncio
import json
import time
import uuid

from aiohttp import web

from ..models.sampling import SamplingParams
from .engine_loop import EngineLoop, GenParams


class ServerState:
    def __init__(self, loop: EngineLoop, tokenizer, model_name: str, max_model_len: int, info: dict | None = None):
        self.loop = loop
        self.tok = tokenizer
        self.model_name = model_name
        self.max_model_len = max_model_len
        self.info = info or {}
        self.t_start = time.time()


def _prompt_ids(st: ServerState, body: dict, chat: bool) -> list[int]:
    if chat:
        text = st.tok.apply_chat_template(body.get("messages") or [])
        return st.tok.encode(text, add_bos=True)
    p = body.get("prompt", "")
    if isinstance(p, list):
        if p and all(isinstance(t, int) for t in p):
            return [int(t) for t in p]
        if len(p) != 1:
            raise web.HTTPBadRequest(text=json.dumps({"error": "batched prompts: send one prompt per request"}),
                                     content_type="application/json")
        p = p[0]
    return st.tok.encode(str(p), add_bos=True)


def _params(st: ServerState, body: dict, n_prompt: int, chat: bool = False) -> tuple[GenParams, list[str]]:
    mt = body.get("max_completion_tokens") or body.get("max_tokens") or body.get("max_new_tokens") or 256
    mt = int(mt)
    if mt < 1:
        raise web.HTTPBadRequest(text=json.dumps({"error": "max_tokens must be >= 1"}), content_type="application/json")
    if n_prompt + mt > st.max_model_len:
        raise web.HTTPBadRequest(
            text=json.dumps({"error": f"prompt ({n_prompt}) + max_tokens ({mt}) exceeds max_model_len "
                                      f"({st.max_model_len})"}), content_type="application/json")
    stop = body.get("stop") or []
    if isinstance(stop, str):
        stop = [stop]
    stop_ids = tuple(int(t) for t in (body.get("stop_token_ids") or []))
    temp = body.get("temperature")
    temp = 0.0 if temp is None else float(temp)
    if temp < 0:
        raise web.HTTPBadRequest(text=json.dumps({"error": "temperature must be >= 0"}),
                                 content_type="application/json")
    for key in ("n", "best_of"):
        if body.get(key) is not None and int(body[key]) != 1:
            raise web.HTTPBadRequest(text=json.dumps({"error": f"{key} > 1 is not supported (one choice per request)"}),
                                     content_type="application/json")
    try:
        top_p = 1.0 if body.get("top_p") is None else float(body["top_p"])
        top_k = 0 if body.get("top_k") is None else int(body["top_k"])
        lp = _logprobs_field(body, chat)
        seed = None if body.get("seed") is None else int(body["seed"])
        sp = SamplingParams(temp, max(top_k, 0), top_p, lp, seed)     # top_k -1 (vLLM's "off") counts as 0
    except (TypeError, ValueError) as e:
        raise web.HTTPBadRequest(text=json.dumps({"error": str(e)}), content_type="application/json") from None
    return (GenParams(mt, bool(body.get("ignore_eos", False)), stop_ids, temp, sp.top_k, sp.top_p, sp.logprobs,
                      sp.seed),
            [s for s in stop if s])


def _logprobs_field(body: dict, chat: bool) -> int | None:
    """Alternatives per token the request asks for (None: no log-probabilities).
    Chat: ``logprobs`` is a switch and ``top_logprobs`` the count; completions:
    ``logprobs`` is the count."""
    if chat:
        if not body.get("logprobs"):
            if body.get("top_logprobs"):
                raise ValueError("top_logprobs needs logprobs: true")
            return None
        return int(body.get("top_logprobs") or 0)
    v = body.get("logprobs")
    if v is None or v is False:
        return None
    return int(v)


def _lp_entry(st: "ServerState", piece: str, lp: dict, chat: bool):
    """One token's log-probability record in the chat layout (the completions
    layout is assembled from the same values by :func:`_completion_logprobs`)."""
    alts = [(st.tok.decode_token(t), v) for t, v in lp["top"]]
    if chat:
        return {"token": piece, "logprob": lp["logprob"], "bytes": list(piece.encode("utf-8")),
                "top_logprobs": [{"token": a, "logprob": v, "bytes": list(a.encode("utf-8"))} for a, v in alts]}
    return piece, lp["logprob"], alts


def _completion_logprobs(entries: list, offset0: int) -> dict:
    tokens, lps, tops, offs = [], [], [], []
    off = offset0
    for piece, v, alts in entries:
        tokens.append(piece)
        lps.append(v)
        tops.append({a: w for a, w in alts})
        offs.append(off)
        off += len(piece)
    return {"tokens": tokens, "token_logprobs": lps, "top_logprobs": tops, "text_offset": offs}


def _err(code: int, msg: str) -> web.Response:
    return web.json_response({"error": {"message": msg, "code": code}}, status=code)


async def _generate(st: ServerState, request: web.Request, chat: bool):
    try:
        body = await request.json()
    except Exception as e:  # noqa: BLE001
        return _err(400, f"invalid JSON: {e}")
    try:
        ids = _prompt_ids(st, body, chat)
        params, stops = _params(st, body, len(ids), chat)
    except web.HTTPBadRequest as e:
        return web.Response(status=400, text=e.text, content_type="application/json")
    if not st.loop.healthy:
        return _err(503, f"engine unhealthy: {st.loop.error}")
    stream = bool(body.get("stream", False))
    rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:16]
    created = int(time.time())
    ts = st.loop.submit(ids, params)
    out_ids: list[int] = []
    text = ""
    finish = None
    want_lp = params.logprobs is not None
    lp_entries: list = []        # per emitted token (chat records, or (piece, lp, alts) for completions)

    def chunk_obj(piece: str | None, fin: str | None, lpe=None) -> dict:
        if chat:
            delta = {} if piece is None else {"content": piece}
            if piece is not None and not out_ids[:-1]:
                delta["role"] = "assistant"
            ch = {"index": 0, "delta": delta, "finish_reason": fin}
            if want_lp:
                ch["logprobs"] = {"content": [lpe]} if lpe is not None else None
            return {"id": rid, "object": "chat.completion.chunk", "created": created, "model": st.model_name,
                    "choices": [ch]}
        lpo = _completion_logprobs([lpe], len(text) - len(piece or "")) if lpe is not None else None
        return {"id": rid, "object": "text_completion", "created": created, "model": st.model_name,
                "choices": [{"index": 0, "text": piece or "", "finish_reason": fin, "logprobs": lpo}]}

    resp = None
    if stream:
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
        await resp.prepare(request)
    try:
        while True:
            kind, val = await ts.q.get()
            if kind == "error":
                if resp is None:
                    return _err(500 if ts.req is not None else 400, val)
                await resp.write(f"data: {json.dumps({'error': {'message': val}})}\n\n".encode())
                finish = "error"
                break
            if kind == "done":
                finish = "stop" if val == "stop" else ("length" if val == "length" else val)
                break
            tok, lp = int(val[0]), val[1]
            out_ids.append(tok)
            if tok == st.tok.eos_token_id and not params.ignore_eos:
                continue
            piece = st.tok.decode_token(tok)
            if stops:
                cand = text + piece
                hit = min((cand.find(s) for s in stops if s in cand), default=-1)
                if hit >= 0:
                    piece = cand[:hit][len(text):]
                    text = cand[:hit]
                    st.loop.cancel(ts)
                    lpe = _lp_entry(st, piece, lp, chat) if (want_lp and lp is not None and piece) else None
                    if lpe is not None:
                        lp_entries.append(lpe)
                    if resp is not None and piece:
                        await resp.write(f"data: {json.dumps(chunk_obj(piece, None, lpe))}\n\n".encode())
                    finish = "stop"
                    # drain until the engine confirms the cancel
                    while True:
                        k2, _ = await ts.q.get()
                        if k2 in ("done", "error"):
                            break
                    break
            lpe = _lp_entry(st, piece, lp, chat) if (want_lp and lp is not None) else None
            if lpe is not None:
                lp_entries.append(lpe)
            text += piece
            if resp is not None:
                await resp.write(f"data: {json.dumps(chunk_obj(piece, None, lpe))}\n\n".encode())
    except (asyncio.CancelledError, ConnectionResetError):
        st.loop.cancel(ts)
        raise
    usage = {"prompt_tokens": len(ids), "completion_tokens": len(out_ids), "total_tokens": len(ids) + len(out_ids)}
    if resp is not None:
        last = chunk_obj(None, finish)
        last["usage"] = usage
        await resp.write(f"data: {json.dumps(last)}\n\n".encode())
        await resp.write(b"data: [DONE]\n\n")
        await resp.write_eof()
        return resp
    if chat:
        choice = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": finish}
        if want_lp:
            choice["logprobs"] = {"content": lp_entries}
        obj = "chat.completion"
    else:
        choice = {"index": 0, "text": text, "finish_reason": finish,
                  "logprobs": _completion_logprobs(lp_entries, 0) if want_lp else None}
        obj = "text_completion"
    req = ts.req
    metrics = {"ttft_s": (req.t_first_token - req.t_arrival) if req and req.t_first_token else None,
               "e2e_s": (req.t_done - req.t_arrival) if req and req.t_done else None}
    return web.json_response({"id": rid, "object": obj, "created": created, "model": st.model_name,
                              "choices": [choice], "usage": usage, "x_metrics": metrics})


def build_app(st: ServerState) -> web.Application:
    app = web.Application(client_max_size=64 * 1024 * 1024)

    async def health(_):
        lp = st.loop
        body = {"status": "ok" if lp.healthy else "unhealthy", "error": lp.error, "model": st.model_name,
                "uptime_s": time.time() - st.t_start, "live_requests": lp.n_live,
                "total_requests": lp.stats["requests"], "total_generated_tokens": lp.stats["generated_tokens"],
                **st.info}
        return web.json_response(body, status=200 if lp.healthy else 503)

    async def models(_):
        return web.json_response({"object": "list", "data": [
            {"id": st.model_name, "object": "model", "created": int(st.t_start), "owned_by": "dsv4-b200",
             "max_model_len": st.max_model_len}]})

    async def tokenize(request):
        body = await request.json()
        if "messages" in body:
            ids = st.tok.encode(st.tok.apply_chat_template(body["messages"]), add_bos=True)
        else:
            ids = st.tok.encode(str(body.get("prompt", "")), add_bos=bool(body.get("add_special_tokens", True)))
        return web.json_response({"count": len(ids), "tokens": ids, "max_model_len": st.max_model_len})

    async def detokenize(request):
        body = await request.json()
        return web.json_response({"prompt": st.tok.decode([int(t) for t in body.get("tokens", [])])})

    async def metrics(_):
        from .metrics import render_prometheus
        return web.Response(text=render_prometheus(st), content_type="text/plain", charset="utf-8")

    async def completions(request):
        return await _generate(st, request, chat=False)

    async def chat(request):
        return await _generate(st, request, chat=True)

    app.router.add_get("/health", health)
    app.router.add_get("/v1/models", models)
    app.router.add_get("/metrics", metrics)
    app.router.add_post("/tokenize", tokenize)
    app.router.add_post("/detokenize", detokenize)
    app.router.add_post("/v1/completions", completions)
    app.router.add_post("/v1/chat/completions", chat)
    return app
