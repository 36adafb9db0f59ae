"""OpenAI-compatible HTTP server.

Endpoints (the union of the reference's ``tpu-v7x/deepseek_v41/server.py``
and what its sweep client asks of vLLM, ``kernel-optimizations-recipe/
scripts/benchmark_sweep.py:70-125``):

  GET  /health                 status, model, device, totals (503 when the engine is unhealthy)
  GET  /v1/models              the served model id
  GET  /metrics                Prometheus text: requests, tokens, step time, batch, TTFT, slots
  POST /tokenize               {"prompt"} or {"messages"} -> {"count", "tokens", "max_model_len"}
  POST /detokenize             {"tokens"} -> {"prompt"}
  POST /v1/completions         prompt (text | ids | a list of either), n, max_tokens, stream, ignore_eos, stop
  POST /v1/chat/completions    messages, n, max_tokens / max_completion_tokens, stream, stop

Decoding: ``temperature`` 0 (the default when the field is absent, and what
every reference benchmark sends) is greedy; ``temperature`` > 0 samples
softmax(logits / T) on the device by the Gumbel-max rule, restricted by
``top_k`` (> 0) and ``top_p`` (< 1) when given; ``seed`` makes the samples a
function of (seed, position) only, so a seeded request repeats its output.
``logprobs`` (completions: the number of alternatives, 0-20; chat:
``logprobs: true`` with ``top_logprobs`` 0-20) returns each generated token's
log-probability under the raw logits and its most likely alternatives, in the
OpenAI response layouts.  ``n`` choices per prompt (and a list of prompts)
run as separate engine requests that share the engine's steps; ``best_of``
is accepted only equal to ``n``.  A request the engine cannot serve is refused
with 400 (top-k / top-p / logprobs on the tensor-parallel head, logprobs or
temperature under speculative decoding).
Streaming sends one SSE event per generated token and ends with
``data: [DONE]``; usage rides on the last finish chunk, or with
``stream_options: {"include_usage": true}`` in one more chunk with no choices.
``echo`` (completions) puts the prompt's text before the completion.  A
client that disconnects cancels its request.

Run: ``python -m dsv4_flash_deployment_b200.serving --config v4-flash --port 8000``.
"""

from __future__ import annotations

import asyncio
import dataclasses
import json
import time
import uuid

from aiohttp import web

from ..models.sampling import SamplingParams
from .engine_loop import EngineLoop, GenParams


class ServerState:
    """``api_key``: when set, every ``/v1/*``, ``/tokenize`` and ``/detokenize``
    request must carry ``Authorization: Bearer <api_key>`` (vLLM's ``--api-key``);
    ``/health`` and ``/metrics`` stay open for probes and scrapers."""

    def __init__(self, loop: EngineLoop, tokenizer, model_name: str, max_model_len: int, info: dict | None = None,
                 api_key: str | None = None):
        self.api_key = api_key
        self.loop = loop
        self.tok = tokenizer
        self.model_name = model_name
        self.max_model_len = max_model_len
        self.info = info or {}
        self.t_start = time.time()


MAX_CHOICES = 64   # prompts x n per request


def _prompt_ids(st: ServerState, body: dict, chat: bool) -> list[list[int]]:
    """Token ids of every prompt: chat messages (one), or a completions ``prompt``
    that is a string, a list of token ids, or a list of either (a batch)."""
    if chat:
        text = st.tok.apply_chat_template(body.get("messages") or [])
        return [st.tok.encode(text, add_bos=True)]
    p = body.get("prompt", "")
    if isinstance(p, list) and p and all(isinstance(t, int) for t in p):
        return [[int(t) for t in p]]
    items = p if isinstance(p, list) else [p]
    if not items or len(items) > MAX_CHOICES:
        raise web.HTTPBadRequest(text=json.dumps({"error": f"between 1 and {MAX_CHOICES} prompts per request"}),
                                 content_type="application/json")
    out = []
    for it in items:
        if isinstance(it, list) and all(isinstance(t, int) for t in it):
            out.append([int(t) for t in it])
        else:
            out.append(st.tok.encode(str(it), add_bos=True))
    if any(not ids for ids in out):
        raise web.HTTPBadRequest(text=json.dumps({"error": "empty prompt"}), content_type="application/json")
    return out


def _n_choices(body: dict) -> int:
    """``n`` choices per prompt; ``best_of`` is accepted only as n (no ranking)."""
    try:
        n = 1 if body.get("n") is None else int(body["n"])
        best_of = body.get("best_of")
        if not 1 <= n <= MAX_CHOICES or (best_of is not None and int(best_of) != n):
            raise ValueError
    except (TypeError, ValueError):
        raise web.HTTPBadRequest(text=json.dumps({"error": f"n must be 1..{MAX_CHOICES}; best_of, if given, "
                                                           "must equal n"}), content_type="application/json") from None
    return n


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


class _Choice:
    """One generated sequence of a request: its token stream, the text after the
    EOS and stop-string rules, the token count and the log-probability records."""

    def __init__(self, index: int, n_prompt: int, ts, params: GenParams, stops: list[str]):
        self.index, self.n_prompt, self.ts, self.params, self.stops = index, n_prompt, ts, params, stops
        self.text = ""
        self.detok = None             # the tokenizer's streaming decoder (set by _consume)
        self.out_ids: list[int] = []
        self.finish: str | None = None
        self.error: str | None = None
        self.lp_entries: list = []   # chat records, or (piece, lp, alts) for completions


async def _consume(st: ServerState, ch: _Choice, chat: bool, emit=None) -> None:
    """Reads the choice's stream to its end; ``emit(ch, piece, lp_record)`` is awaited
    for every piece of text (streaming responses)."""
    want_lp = ch.params.logprobs is not None
    ts = ch.ts
    mk = getattr(st.tok, "stream_decoder", None)
    ch.detok = mk() if mk is not None else None
    while True:
        kind, val = await ts.q.get()
        if kind == "error":
            ch.error, ch.finish = val, "error"
            return
        if kind == "done":
            ch.finish = "stop" if val == "stop" else ("length" if val == "length" else val)
            tail = ch.detok.flush() if ch.detok is not None else ""
            if tail:
                ch.text += tail
                if emit is not None:
                    await emit(ch, tail, None)
            return
        tok, lp = int(val[0]), val[1]
        ch.out_ids.append(tok)
        if tok == st.tok.eos_token_id and not ch.params.ignore_eos:
            continue
        piece = ch.detok.push(tok) if ch.detok is not None else st.tok.decode_token(tok)
        if not piece and lp is None:
            continue                  # the token's text is still incomplete: nothing to send yet
        if ch.stops:
            cand = ch.text + piece
            hit = min((cand.find(s) for s in ch.stops if s in cand), default=-1)
            if hit >= 0:
                piece = cand[:hit][len(ch.text):]
                ch.text = cand[:hit]
                st.loop.cancel(ts)
                lpe = _lp_entry(st, piece, lp, chat) if (want_lp and lp is not None and piece) else None
                if lpe is not None:
                    ch.lp_entries.append(lpe)
                if emit is not None and piece:
                    await emit(ch, piece, lpe)
                ch.finish = "stop"
                while True:          # drain until the engine confirms the cancel
                    k2, _ = await ts.q.get()
                    if k2 in ("done", "error"):
                        return
        lpe = _lp_entry(st, piece, lp, chat) if (want_lp and lp is not None) else None
        if lpe is not None:
            ch.lp_entries.append(lpe)
        ch.text += piece
        if emit is not None:
            await emit(ch, piece, lpe)


async def _generate(st: ServerState, request: web.Request, chat: bool):
    """One request: every prompt (completions take a list) times ``n`` choices, each
    its own engine request (a seeded request's choice j uses seed + j); choice
    index = prompt index * n + j."""
    try:
        body = await request.json()
    except Exception as e:  # noqa: BLE001
        return _err(400, f"invalid JSON: {e}")
    try:
        prompts = _prompt_ids(st, body, chat)
        params, stops = _params(st, body, max(len(p) for p in prompts), chat)
        n = _n_choices(body)
    except web.HTTPBadRequest as e:
        return web.Response(status=400, text=e.text, content_type="application/json")
    if not st.loop.healthy:
        return _err(503, f"engine unhealthy: {st.loop.error}")
    if st.loop.draining:
        return _err(503, "the server is shutting down")
    stream = bool(body.get("stream", False))
    rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:16]
    created = int(time.time())
    want_lp = params.logprobs is not None
    choices = []
    for pi, ids in enumerate(prompts):
        for j in range(n):
            pj = params if params.seed is None or j == 0 else dataclasses.replace(params, seed=params.seed + j)
            choices.append(_Choice(pi * n + j, len(ids), st.loop.submit(ids, pj), pj, stops))

    def chunk_obj(ch: _Choice, piece: str | None, fin: str | None, lpe=None) -> dict:
        if chat:
            delta = {} if piece is None else {"content": piece}
            if piece is not None and not ch.out_ids[:-1]:
                delta["role"] = "assistant"
            c = {"index": ch.index, "delta": delta, "finish_reason": fin}
            if want_lp:
                c["logprobs"] = {"content": [lpe]} if lpe is not None else None
            return {"id": rid, "object": "chat.completion.chunk", "created": created, "model": st.model_name,
                    "choices": [c]}
        lpo = _completion_logprobs([lpe], len(ch.text) - len(piece or "")) if lpe is not None else None
        return {"id": rid, "object": "text_completion", "created": created, "model": st.model_name,
                "choices": [{"index": ch.index, "text": piece or "", "finish_reason": fin, "logprobs": lpo}]}

    resp = None
    emit = None
    if stream:
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
        await resp.prepare(request)

        # the per-token event without log-probabilities, past the first chunk of a
        # chat choice (which carries the role), is the same text around the piece:
        # built from a fixed head and tail instead of encoding a dict per token
        head = json.dumps({"id": rid, "object": "chat.completion.chunk" if chat else "text_completion",
                           "created": created, "model": st.model_name})[:-1]
        tail = ('}, "finish_reason": null}]}\n\n' if chat else ', "finish_reason": null, "logprobs": null}]}\n\n')

        async def emit(ch, piece, lpe):
            if lpe is None and not want_lp and not (chat and not ch.out_ids[:-1]):
                key = '"delta": {"content": ' if chat else '"text": '
                line = f'data: {head}, "choices": [{{"index": {ch.index}, {key}{json.dumps(piece)}{tail}'
            else:
                line = f"data: {json.dumps(chunk_obj(ch, piece, None, lpe))}\n\n"
            await resp.write(line.encode())
    try:
        await asyncio.gather(*(_consume(st, ch, chat, emit) for ch in choices))
    except (asyncio.CancelledError, ConnectionResetError):
        for ch in choices:
            st.loop.cancel(ch.ts)
        raise
    failed = [ch for ch in choices if ch.error is not None]
    if failed and resp is None:
        for ch in choices:
            st.loop.cancel(ch.ts)
        refused = any(ch.ts.req is None for ch in failed)    # the engine refused it before it started
        return _err(400 if refused else 500, failed[0].error)
    n_out = sum(len(ch.out_ids) for ch in choices)
    n_in = sum(len(p) for p in prompts)
    usage = {"prompt_tokens": n_in, "completion_tokens": n_out, "total_tokens": n_in + n_out}
    if resp is not None:
        # stream_options.include_usage: usage in one more chunk with no choices (the
        # OpenAI layout); otherwise on the last finish chunk
        usage_chunk = bool((body.get("stream_options") or {}).get("include_usage"))
        for ch in choices:
            if ch.error is not None:
                await resp.write(f"data: {json.dumps({'error': {'message': ch.error}})}\n\n".encode())
            last = chunk_obj(ch, None, ch.finish)
            if ch is choices[-1] and not usage_chunk:
                last["usage"] = usage
            await resp.write(f"data: {json.dumps(last)}\n\n".encode())
        if usage_chunk:
            u = {"id": rid, "object": "chat.completion.chunk" if chat else "text_completion", "created": created,
                 "model": st.model_name, "choices": [], "usage": usage}
            await resp.write(f"data: {json.dumps(u)}\n\n".encode())
        await resp.write(b"data: [DONE]\n\n")
        await resp.write_eof()
        return resp
    out = []
    for ch in choices:
        if chat:
            c = {"index": ch.index, "message": {"role": "assistant", "content": ch.text}, "finish_reason": ch.finish}
            if want_lp:
                c["logprobs"] = {"content": ch.lp_entries}
        else:
            # echo: the prompt's text before the completion (its tokens carry no log-probabilities)
            pre = st.tok.decode(prompts[ch.index // n]) if body.get("echo") else ""
            c = {"index": ch.index, "text": pre + ch.text, "finish_reason": ch.finish,
                 "logprobs": _completion_logprobs(ch.lp_entries, len(pre)) if want_lp else None}
        out.append(c)
    req = choices[0].ts.req
    metrics = {"ttft_s": (req.t_first_token - req.t_arrival) if req and req.t_first_token else None,
               "e2e_s": (req.t_done - req.t_arrival) if req and req.t_done else None}
    return web.json_response({"id": rid, "object": "chat.completion" if chat else "text_completion",
                              "created": created, "model": st.model_name, "choices": out, "usage": usage,
                              "x_metrics": metrics})


OPEN_PATHS = ("/health", "/metrics")


def build_app(st: ServerState) -> web.Application:
    @web.middleware
    async def auth(request, handler):
        if st.api_key and request.path not in OPEN_PATHS:
            import hmac

            got = request.headers.get("Authorization", "")
            if not hmac.compare_digest(got.encode(), f"Bearer {st.api_key}".encode()):
                return _err(401, "missing or wrong API key")
        return await handler(request)

    app = web.Application(client_max_size=64 * 1024 * 1024, middlewares=[auth])

    async def health(_):
        lp = st.loop
        status = "unhealthy" if not lp.healthy else ("draining" if lp.draining else "ok")
        body = {"status": status, "error": lp.error, "model": st.model_name,
                "uptime_s": time.time() - st.t_start, "live_requests": lp.n_live,
                "total_requests": lp.stats["requests"], "total_generated_tokens": lp.stats["generated_tokens"],
                **st.info}
        return web.json_response(body, status=200 if status == "ok" else 503)

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
