"""FastAPI application over an AsyncEngine."""
from __future__ import annotations

import json
import time
import uuid

from .. import __version__
from ..obs.metrics import METRICS
from ..runtime.engine import SamplingParams
from ..text.chat import apply_chat_template, chat_ids
from ..text.tokenizer import IncrementalDecoder

MAX_BODY = 32 << 20

try:  # FastAPI resolves handler annotations from module globals
    from fastapi import Request
except ImportError:  # pragma: no cover
    Request = None


def _chat(tokenizer):
    """The tokenizer's own chat template when it has one (checkpoint directories), else ChatML."""
    return getattr(tokenizer, "apply_chat_template", apply_chat_template)


def _chat_ids(tokenizer, msgs, system=None) -> list[int]:
    return chat_ids(tokenizer, msgs, system)


def _err(status: int, typ: str, msg: str):
    from fastapi.responses import JSONResponse
    return JSONResponse(status_code=status, content={"error": {"type": typ, "message": msg}})


def _params(body: dict, default_max: int = 16, stop_ids: tuple = ()) -> SamplingParams:
    """OpenAI / Anthropic request fields -> SamplingParams; generation stops at the tokenizer's
    stop ids (end of sequence / end of turn) unless the request sets `ignore_eos`."""
    stop = tuple(body.get("stop_token_ids") or ()) + (() if body.get("ignore_eos") else tuple(stop_ids))
    return SamplingParams(max_tokens=int(body.get("max_tokens", body.get("max_completion_tokens", default_max))),
                          temperature=float(body.get("temperature", 1.0 if "temperature" not in body else
                                                     body["temperature"])),
                          top_k=int(body.get("top_k", 0)), top_p=float(body.get("top_p", 1.0)),
                          seed=body.get("seed"), stop_token_ids=tuple(stop), constraint=_constraint(body),
                          repetition_penalty=float(body.get("repetition_penalty", 1.0)),
                          frequency_penalty=float(body.get("frequency_penalty", 0.0)),
                          presence_penalty=float(body.get("presence_penalty", 0.0)),
                          logit_bias={int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()} or None,
                          logprobs=_logprobs_k(body))


def _logprobs_k(body: dict):
    """Chat `logprobs: true` (+ `top_logprobs: n`) or completions `logprobs: n` -> alternatives
    per token (None when not asked)."""
    lp = body.get("logprobs")
    if lp is True:
        n = body.get("top_logprobs") or 0
        return n if isinstance(n, int) and not isinstance(n, bool) else -1  # -1: rejected by the engine
    if isinstance(lp, int) and not isinstance(lp, bool):
        return lp
    return None


def _render_logprobs(tokenizer, recs: list, chat: bool) -> dict:
    def tok(t):
        return tokenizer.decode([t])
    if chat:
        return {"content": [{"token": tok(r["token"]), "logprob": r["logprob"],
                             "top_logprobs": [{"token": tok(t), "logprob": v} for t, v in r["top"]]} for r in recs]}
    return {"tokens": [tok(r["token"]) for r in recs], "token_logprobs": [r["logprob"] for r in recs],
            "top_logprobs": [{tok(t): v for t, v in r["top"]} for r in recs]}


def _constraint(body: dict):
    """OpenAI `response_format` json_object / json_schema (any JSON object; the schema itself
    is not enforced) and the `guided_choice` list extension -> a decoding constraint."""
    rf = body.get("response_format") or {}
    if isinstance(rf, dict) and rf.get("type") in ("json_object", "json_schema"):
        return {"type": "json"}
    if body.get("guided_choice"):
        return {"choices": [str(c) for c in body["guided_choice"]]}
    return body.get("constraint")


def build_app(aeng, tokenizer, model_id: str = "syntropy", bench_api: bool = True):
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="syntropy_b200")
    vocab = aeng.engine.cfg.vocab
    aeng.engine.set_tokenizer(tokenizer)  # vocabulary bytes for constrained requests

    async def _body(req: Request):
        raw = await req.body()
        if len(raw) > MAX_BODY:
            return None, _err(413, "request_too_large", f"body over {MAX_BODY} bytes")
        try:
            return json.loads(raw or b"{}"), None
        except json.JSONDecodeError as e:
            return None, _err(400, "invalid_request", f"invalid JSON: {e}")

    def _check_ids(ids, field_name="tokens"):
        for i, t in enumerate(ids):
            if not isinstance(t, int) or not 0 <= t < vocab:
                return _err(400, "token_id_out_of_range", f"{field_name}[{i}]={t} outside [0, {vocab})")
        return None

    @app.get("/healthz")
    async def healthz():
        return {"status": "ok"}

    @app.get("/readyz")
    async def readyz():
        if not aeng.ready:
            return JSONResponse(status_code=503, content={"status": "starting"})
        return {"status": "ready"}

    @app.get("/v1/syntropy/version")
    async def version():
        return {"version": __version__, "engine": "syntropy_b200", "arch": "sm_100a"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_id, "object": "model", "owned_by": "syntropy_b200",
                                            "created": 0}]}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(METRICS.prometheus())

    # ---------------------------------------------------------------- native generate
    @app.post("/v1/syntropy/generate")
    async def native_generate(req: Request):
        if not bench_api:
            return _err(404, "unsupported_endpoint", "native generate is disabled (debug.bench_api)")
        body, err = await _body(req)
        if err:
            return err
        allowed = {"model", "tokens", "sampling", "stream", "return_tokens", "prompt", "messages", "constraint"}
        unknown = set(body) - allowed
        if unknown:
            return _err(400, "invalid_request", f"unknown fields {sorted(unknown)}")
        ids = body.get("tokens")
        if ids is None and body.get("prompt") is None and body.get("messages"):
            ids = _chat_ids(tokenizer, body["messages"])
        if ids is None:
            text = body.get("prompt")
            if text is None:
                return _err(400, "invalid_request", "one of tokens, prompt or messages is required")
            ids = tokenizer.encode(text)
        e = _check_ids(ids)
        if e:
            return e
        sp = body.get("sampling") or {}
        params = SamplingParams(max_tokens=int(sp.get("max_tokens", 16)), temperature=float(sp.get("temperature", 0.0)),
                                top_k=int(sp.get("top_k", 0)), top_p=float(sp.get("top_p", 1.0)), seed=sp.get("seed"),
                                constraint=body.get("constraint"))
        ret_tokens = bool(body.get("return_tokens", False))
        seq = uuid.uuid4().hex[:16]

        async def gen():
            n = 0
            dec = IncrementalDecoder(tokenizer)
            async for ev in aeng.generate(list(ids), params):
                if ev.kind == "started":
                    line = {"event": "started", "sequence": seq, "prompt_tokens": len(ids), "cached_tokens": 0}
                elif ev.kind == "tokens":
                    line = {"event": "text", "text": dec.push(ev.tokens)}
                    if ret_tokens:
                        line["tokens"] = ev.tokens
                elif ev.kind == "done":
                    line = {"event": "done", "finish_reason": ev.finish_reason, "usage": ev.usage,
                            "timings": ev.timings}
                else:
                    line = {"event": "error", "error": {"type": "invalid_request" if ev.status == 400 else "internal",
                                                        "message": ev.error}}
                line["id"] = f"{seq}:{n}"
                n += 1
                yield json.dumps(line) + "\n"

        return StreamingResponse(gen(), media_type="application/x-ndjson")

    # ---------------------------------------------------------------- OpenAI
    async def _openai(req: Request, chat: bool):
        body, err = await _body(req)
        if err:
            return err
        if chat:
            msgs = body.get("messages")
            if not isinstance(msgs, list) or not msgs:
                return _err(400, "invalid_request", "messages must be a non-empty list")
            ids = _chat_ids(tokenizer, msgs)
        else:
            p = body.get("prompt")
            if isinstance(p, list) and p and isinstance(p[0], int):
                ids = p
            elif isinstance(p, str):
                ids = tokenizer.encode(p)
            else:
                return _err(400, "invalid_request", "prompt must be a string or a list of token ids")
        e = _check_ids(ids, "prompt")
        if e:
            return e
        params = _params(body, stop_ids=tuple(getattr(tokenizer, "stop_token_ids", ()) or ()))
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if body.get("stream"):
            async def sse():
                dec = IncrementalDecoder(tokenizer)
                async for ev in aeng.generate(list(ids), params):
                    if ev.kind == "tokens":
                        t = dec.push(ev.tokens)
                        choice = ({"index": 0, "delta": {"content": t}, "finish_reason": None} if chat else
                                  {"index": 0, "text": t, "finish_reason": None})
                        if ev.logprobs:
                            choice["logprobs"] = _render_logprobs(tokenizer, ev.logprobs, chat)
                        yield "data: " + json.dumps({"id": rid, "object": obj + ".chunk", "created": created,
                                                     "model": model_id, "choices": [choice]}) + "\n\n"
                    elif ev.kind == "done":
                        choice = ({"index": 0, "delta": {}, "finish_reason": ev.finish_reason} if chat else
                                  {"index": 0, "text": "", "finish_reason": ev.finish_reason})
                        yield "data: " + json.dumps({"id": rid, "object": obj + ".chunk", "created": created,
                                                     "model": model_id, "choices": [choice],
                                                     "usage": ev.usage}) + "\n\n"
                    elif ev.kind == "error":
                        yield "data: " + json.dumps({"error": {"message": ev.error}}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        toks, usage, reason, lps = [], None, None, None
        async for ev in aeng.generate(list(ids), params):
            if ev.kind == "tokens":
                toks += ev.tokens
            elif ev.kind == "done":
                usage, reason, lps = ev.usage, ev.finish_reason, ev.logprobs
            elif ev.kind == "error":
                return _err(ev.status, "invalid_request" if ev.status == 400 else "internal", ev.error)
        text = tokenizer.decode(toks)
        choice = ({"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": reason} if chat
                  else {"index": 0, "text": text, "finish_reason": reason})
        if lps is not None:
            choice["logprobs"] = _render_logprobs(tokenizer, lps, chat)
        if usage:
            usage["total_tokens"] = usage["prompt_tokens"] + usage["completion_tokens"]
        return {"id": rid, "object": obj, "created": created, "model": model_id, "choices": [choice], "usage": usage}

    @app.post("/v1/completions")
    async def completions(req: Request):
        return await _openai(req, chat=False)

    @app.post("/v1/chat/completions")
    async def chat_completions(req: Request):
        return await _openai(req, chat=True)

    # ---------------------------------------------------------------- Anthropic
    @app.post("/v1/messages")
    async def messages(req: Request):
        body, err = await _body(req)
        if err:
            return err
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            return _err(400, "invalid_request_error", "messages must be a non-empty list")
        if "max_tokens" not in body:
            return _err(400, "invalid_request_error", "max_tokens is required")
        sysm = body.get("system")
        if isinstance(sysm, list):
            sysm = "".join(b.get("text", "") for b in sysm)
        ids = _chat_ids(tokenizer, msgs, system=sysm)
        params = _params(body, stop_ids=tuple(getattr(tokenizer, "stop_token_ids", ()) or ()))
        mid = "msg_" + uuid.uuid4().hex[:24]
        stop_map = {"length": "max_tokens", "stop": "end_turn", "cancelled": "end_turn"}
        if body.get("stream"):
            async def sse():
                dec = IncrementalDecoder(tokenizer)
                yield "event: message_start\ndata: " + json.dumps({"type": "message_start", "message": {
                    "id": mid, "type": "message", "role": "assistant", "model": model_id, "content": [],
                    "stop_reason": None, "usage": {"input_tokens": len(ids), "output_tokens": 0}}}) + "\n\n"
                yield "event: content_block_start\ndata: " + json.dumps(
                    {"type": "content_block_start", "index": 0, "content_block": {"type": "text", "text": ""}}) + "\n\n"
                async for ev in aeng.generate(list(ids), params):
                    if ev.kind == "tokens":
                        yield "event: content_block_delta\ndata: " + json.dumps(
                            {"type": "content_block_delta", "index": 0,
                             "delta": {"type": "text_delta", "text": dec.push(ev.tokens)}}) + "\n\n"
                    elif ev.kind == "done":
                        yield "event: content_block_stop\ndata: " + json.dumps(
                            {"type": "content_block_stop", "index": 0}) + "\n\n"
                        yield "event: message_delta\ndata: " + json.dumps(
                            {"type": "message_delta", "delta": {"stop_reason": stop_map.get(ev.finish_reason,
                                                                                           "end_turn")},
                             "usage": {"output_tokens": ev.usage["completion_tokens"]}}) + "\n\n"
                        yield "event: message_stop\ndata: " + json.dumps({"type": "message_stop"}) + "\n\n"
                    elif ev.kind == "error":
                        yield "event: error\ndata: " + json.dumps({"type": "error", "error": {
                            "type": "api_error", "message": ev.error}}) + "\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        toks, usage, reason = [], None, None
        async for ev in aeng.generate(list(ids), params):
            if ev.kind == "tokens":
                toks += ev.tokens
            elif ev.kind == "done":
                usage, reason = ev.usage, ev.finish_reason
            elif ev.kind == "error":
                return _err(ev.status, "invalid_request_error" if ev.status == 400 else "api_error", ev.error)
        return {"id": mid, "type": "message", "role": "assistant", "model": model_id,
                "content": [{"type": "text", "text": tokenizer.decode(toks)}],
                "stop_reason": stop_map.get(reason, "end_turn"), "stop_sequence": None,
                "usage": {"input_tokens": usage["prompt_tokens"], "output_tokens": usage["completion_tokens"]}}

    return app
