"""Async client of the server's session routes: a multi-turn conversation holds one server session, so each new
turn prefills only the text added since the previous one (the reference's `_SessionEndpoint`,
flashnext/kaggle/code_dataset/repl_solve.py:1556-1760).

Protocol: the first turn opens ``POST /arc/session`` (NDJSON stream, ``keep``); later turns ``push`` the pending
token of the previous chunk followed by the new tokens; a chunk that ends at its token budget is continued by
pushing back its last token; a 409 (context full) ends the session and the turn returns with "length".
"""
from __future__ import annotations

import json

import aiohttp


class SessionClient:
    def __init__(self, base: str, tokenizer, rid: str, max_model_len: int, temperature=1.0, top_p=1.0, seed=None,
                 chunk: int = 256, stop_token_ids=()):
        self.base, self.tok, self.rid = base.rstrip("/"), tokenizer, rid
        self.M = max_model_len
        self.samp = {"temperature": temperature, "top_p": top_p}
        if seed is not None:
            self.samp["seed"] = seed
        self.chunk = chunk
        self.stop = list(stop_token_ids)
        self.http = None
        self.resp = None
        self.lines = None
        self.known = ""       # conversation text the server holds
        self.last_id = None   # pending (unfed) token
        self.held = 0

    async def _lines(self):
        async for raw in self.resp.content:
            line = raw.strip()
            if line:
                yield json.loads(line)

    async def close(self):
        if self.resp is not None:
            try:
                async with self.http.post(self.base + "/arc/session/close", json={"rid": self.rid}) as r:
                    await r.read()
            except aiohttp.ClientError:
                pass
            self.resp.release()
            self.resp = None
        if self.http is not None:
            await self.http.close()
            self.http = None

    @staticmethod
    def render(messages) -> str:
        return "".join(f"<|{m['role']}|>\n{m['content']}\n" for m in messages) + "<|assistant|>\n"

    async def __call__(self, messages, max_tokens: int) -> str:
        if self.http is None:
            self.http = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None, sock_read=600))
        prompt = self.render(messages)
        extend = self.resp is not None and prompt.startswith(self.known) and self.last_id is not None
        ids_out, text = [], ""
        if extend:
            ids = [self.last_id] + self.tok.encode(prompt[len(self.known):])
            if self.held + len(ids) >= self.M - 1:
                await self.close()
                return ""
            await self._push(ids, min(self.chunk, max_tokens))
        else:
            await self.close()
            self.http = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None, sock_read=600))
            ids = self.tok.encode(prompt)
            if len(ids) >= self.M - 1:
                return ""
            body = {"rid": self.rid, "prompt_ids": ids, "max_tokens": min(self.chunk, max_tokens), "keep": True,
                    "stop_token_ids": self.stop, **self.samp}
            self.resp = await self.http.post(self.base + "/arc/session", json=body)
            if self.resp.status != 200:
                raise RuntimeError(f"session HTTP {self.resp.status}: {(await self.resp.text())[:200]}")
            self.lines = self._lines().__aiter__()
            self.held = len(ids)
        if extend:
            self.held += len(ids)
        while True:
            ev = await self.lines.__anext__()
            if "ids" in ev:
                ids_out += ev["ids"]
                text += ev["text"]
            elif "chunk_end" in ev:
                if ev["chunk_end"] != "length" or ev.get("ctx_full") or len(ids_out) >= max_tokens:
                    break
                ok = await self._push([ids_out[-1]], min(self.chunk, max_tokens - len(ids_out)))
                if not ok:
                    break
            elif "end" in ev:
                self.resp = None
                break
        self.held += len(ids_out) - 1 if ids_out else 0
        self.known = prompt + text
        self.last_id = ids_out[-1] if ids_out else None
        return text

    async def _push(self, ids, max_tokens) -> bool:
        async with self.http.post(self.base + "/arc/session/push",
                                  json={"rid": self.rid, "prompt_ids": ids, "max_tokens": max_tokens, "keep": True,
                                        "stop_token_ids": self.stop, **self.samp}) as r:
            if r.status == 409:
                return False
            if r.status != 200:
                raise RuntimeError(f"push HTTP {r.status}")
            return True
