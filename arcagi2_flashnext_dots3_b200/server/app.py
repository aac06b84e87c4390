"""HTTP API: OpenAI-style completions plus the multi-turn session routes the solver uses.

Routes (the reference serves them from vLLM with its session plugin, flashnext/kaggle/code_dataset/fnext/session/
session_ep.py:35-135, and vLLM's OpenAI server):

* ``GET  /health``                      200 while the engine thread is alive
* ``GET  /v1/models``
* ``POST /v1/completions``              {prompt (text or token ids), max_tokens, temperature, top_p, top_k, seed,
                                        stop, stop_token_ids, logprobs, stream}; ``stream`` answers server-sent events
* ``POST /arc/session``                 {rid, prompt_ids, max_tokens, keep, sampling...} -> NDJSON stream of
                                        {"ids", "text"[, "lp"]}, {"chunk_end", "n"[, "ctx_full"]}, ..., {"end", "n"}
* ``POST /arc/session/push``            {rid, prompt_ids, max_tokens, keep, sampling...} -> {"ok"} | 404 | 409
* ``POST /arc/session/close``           {rid} -> {"ok"}
* ``GET  /arc/session/stats``           counters (sessions, open, pushes, generated, ctx_full, ...)
"""
from __future__ import annotations

import asyncio
import json
import time
import uuid

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse

from .engine_loop import EngineLoop, Session
from ..ops.sampling import SamplingParams


def create_app(engine: EngineLoop, model_name: str = "arcagi2-b200"):
    app = FastAPI()
    app.state.engine = engine

    async def _call(kind, **kw):
        return await asyncio.wrap_future(engine.submit(kind, **kw))

    @app.get("/health")
    async def health():
        return JSONResponse({"ok": engine.healthy}, status_code=200 if engine.healthy else 503)

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model",
                                            "max_model_len": engine.llm.ec.max_model_len}]}

    async def _open(b: dict, oneshot: bool):
        prompt = b.get("prompt_ids", b.get("prompt", ""))
        ids = engine.tok.encode(prompt) if isinstance(prompt, str) else [int(t) for t in prompt]
        sp = SamplingParams.from_request(b)
        s = Session(rid=str(b.get("rid") or uuid.uuid4().hex), events=asyncio.Queue(),
                    loop=asyncio.get_running_loop(), keep=bool(b.get("keep")), oneshot=oneshot,
                    want_lp=b.get("logprobs") is not None)
        code, body = await _call("start", session=s, sp=sp, prompt_ids=ids)
        return s, ids, code, body

    @app.post("/arc/session")
    async def session(req: Request):
        b = await req.json()
        s, ids, code, body = await _open(b, oneshot=False)
        if code != 200:
            return JSONResponse(body, status_code=code)

        async def stream():
            while True:
                ev = await s.events.get()
                yield json.dumps(ev) + "\n"
                if "end" in ev:
                    return
        return StreamingResponse(stream(), media_type="application/x-ndjson")

    @app.post("/arc/session/push")
    async def push(req: Request):
        b = await req.json()
        sp = SamplingParams.from_request(b) if any(k in b for k in ("temperature", "top_p", "top_k")) else None
        code, body = await _call("push", rid=str(b["rid"]), prompt_ids=[int(t) for t in b["prompt_ids"]],
                                 max_tokens=int(b.get("max_tokens", 16)), keep=b.get("keep"), sp=sp,
                                 seed=b.get("seed"))
        return JSONResponse(body, status_code=code)

    @app.post("/arc/session/close")
    async def close(req: Request):
        b = await req.json()
        code, body = await _call("close", rid=str(b["rid"]))
        return JSONResponse(body, status_code=code)

    @app.get("/arc/session/stats")
    async def stats():
        out = {k: int(v) for k, v in engine.stats.items()}
        sched = getattr(engine, "sched", None)
        if sched is not None:   # scheduler counters: admissions, preemptions, idle-session evictions, KV state
            out.update({f"sched_{k}": int(v) for k, v in vars(sched.stats).items()})
            out.update(waiting=len(sched.waiting), running=len(sched.running), idle_sessions=len(sched.idle),
                       kv_blocks_free=int(engine.llm.alloc.n_free()),
                       block_size=int(engine.llm.caches.block_size))
        return JSONResponse(out)

    @app.post("/v1/completions")
    async def completions(req: Request):
        b = await req.json()
        stops = [x for x in (b.get("stop") or []) if x]
        s, ids, code, body = await _open(b, oneshot=True)
        if code != 200:
            return JSONResponse({"error": body.get("error")}, status_code=code)
        cid = f"cmpl-{s.rid}"

        async def events():
            text, toks, lps, finish = "", [], [], None
            while True:
                ev = await s.events.get()
                if "ids" in ev:
                    toks += ev["ids"]
                    lps += ev.get("lp", [])
                    piece = ev["text"]
                    text += piece
                    hit = next((x for x in stops if x in text), None)
                    if hit is not None:
                        cut = text.index(hit)
                        piece = piece[: max(0, len(piece) - (len(text) - cut))]
                        text = text[:cut]
                        finish = "stop"
                        await _call("close", rid=s.rid)
                    yield ("tok", piece)
                    if finish:
                        break
                elif "chunk_end" in ev:
                    finish = finish or ev["chunk_end"]
                elif "end" in ev:
                    finish = finish or ("length" if ev["end"] == "ctx_full" else "stop")
                    break
            yield ("done", (text, toks, lps, finish))

        def choice(text, finish, lps=None):
            c = {"text": text, "index": 0, "finish_reason": finish}
            if lps is not None:
                c["logprobs"] = {"token_logprobs": lps}
            return c

        if b.get("stream"):
            async def sse():
                async for kind, val in events():
                    if kind == "tok":
                        yield "data: " + json.dumps({"id": cid, "object": "text_completion", "model": model_name,
                                                     "choices": [choice(val, None)]}) + "\n\n"
                    else:
                        yield "data: " + json.dumps({"id": cid, "object": "text_completion", "model": model_name,
                                                     "choices": [choice("", val[3])]}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        result = None
        async for kind, val in events():
            if kind == "done":
                result = val
        text, toks, lps, finish = result
        return {"id": cid, "object": "text_completion", "created": int(time.time()), "model": model_name,
                "choices": [choice(text, finish, lps if s.want_lp else None)],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                          "total_tokens": len(ids) + len(toks)}}

    return app
