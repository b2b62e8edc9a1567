"""OpenAI-compatible HTTP API (FastAPI) over an InferencePipeline.

Routes
  inference   POST /v1/completions, /api/generate, /v1/chat/completions (tools, SSE),
              /v1/batch/completions (<= 32 prompts), /api/infer (top logits)
  models      GET /v1/models, /api/models; POST /api/models/load; /api/lora
  operations  GET /health /ready /live /metrics /api/status /api/gpu /api/gpu/info
              /api/system /api/pipeline/status /api/queue/status /api/batcher/stats
              /api/history /api/nodes; POST /api/benchmark; GET /chat, /dashboard
  accounts    POST /api/auth/login, /api/auth/refresh, /api/auth/change-password;
              GET /api/auth/me; GET / POST /api/auth/users (admin)
Protection: JWT access tokens with roles user < ops < admin (serving/auth.py) or the
static bearer token (VRM_API_TOKEN, admin), per-route minimum roles, CORS origin
policy (VRM_CORS_ORIGINS), optional HMAC signatures (VRM_HMAC_SECRET), per-IP rate
limit, body cap, read-only mode, audit log; 400 on validation / context overflow,
401 auth, 403 role or origin, 413 body, 429 queue or rate, 503 circuit open or no
model, 504 timeout.

Reference parity: core/production_api.py:156-1556 (Flask app, routes, SSE, queue
counter, circuit breaker, timeouts), core/api/routes_ops.py:23-375,
core/api/registry.py:16-205.  Flask is not installed in this environment; the same
surface is served with FastAPI/uvicorn.
"""
from __future__ import annotations

import asyncio
import hmac
import json
import os
import time
import uuid
from concurrent.futures import ThreadPoolExecutor
from concurrent.futures import TimeoutError as FutTimeout
from typing import Any, Dict, List, Optional

import torch
from fastapi import FastAPI, Request
from fastapi.responses import HTMLResponse, JSONResponse, PlainTextResponse, Response, StreamingResponse

from ..utils.config import flags
from ..utils.monitor import GPUMonitor, health_report, system_info
from ..utils.observability import METRICS, get_logger
from .auth import Auth, AuthError, CorsPolicy, required_role, role_allows
from .security import (AuditLog, CircuitBreaker, QueueCounter, RateLimiter, ValidationError, startup_checks,
                       validate_generation_params, verify_signature)
from .tool_calls import build_chat_message, build_chat_prompt

log = get_logger("vramancer.api")

PUBLIC = {"/health", "/ready", "/live", "/metrics", "/", "/chat", "/dashboard"}
AUTH_OPEN = {"/api/auth/login", "/api/auth/refresh"}     # credentials travel in the body


def _err(status: int, message: str, etype: str = "invalid_request_error", code: Optional[str] = None):
    return JSONResponse({"error": {"message": message, "type": etype, "code": code}}, status_code=status)


class Registry:
    """Holds the served pipeline (lazy load on first use of a model name)."""

    def __init__(self, pipeline=None):
        self.pipeline = pipeline
        self.loading = False

    def get(self, model: Optional[str] = None):
        if self.pipeline is None and model:
            self.load(model)
        return self.pipeline

    def load(self, model: str, **kw):
        from ..pipeline import InferencePipeline
        self.loading = True
        try:
            if self.pipeline is not None:
                self.pipeline.shutdown()
            self.pipeline = InferencePipeline().load(model, **kw)
        finally:
            self.loading = False
        return self.pipeline


def create_app(pipeline=None, *, model_alias: Optional[str] = None) -> FastAPI:
    app = FastAPI(title="VRAMancer-B200", version="0.1.0")
    reg = Registry(pipeline)
    breaker = CircuitBreaker()
    limiter = RateLimiter(int(flags.VRM_RATE_LIMIT_RPM))
    queue = QueueCounter(int(flags.VRM_MAX_QUEUE))
    audit = AuditLog()
    auth = Auth()
    cors = CorsPolicy()
    if os.environ.get("VRM_DEFAULT_ADMIN_PASS"):
        auth.ensure_default_admin(production=bool(flags.VRM_PRODUCTION))
    app.state.auth, app.state.cors = auth, cors
    # credit ledger for sk-VRAM- keys (VRM_LEDGER_DB names its SQLite file; off when unset)
    ledger = None
    if os.environ.get("VRM_LEDGER_DB"):
        from .ledger import CreditLedger
        ledger = CreditLedger(os.environ["VRM_LEDGER_DB"])
    app.state.ledger = ledger
    executor = ThreadPoolExecutor(max_workers=max(1, int(flags.VRM_MAX_CONCURRENT)) * 8,
                                  thread_name_prefix="vrm-api")
    monitor = GPUMonitor()
    app.state.registry, app.state.breaker, app.state.queue, app.state.audit = reg, breaker, queue, audit
    app.state.executor = executor
    app.state.startup_issues = startup_checks(bool(flags.VRM_PRODUCTION))

    def alias():
        p = reg.pipeline
        return model_alias or flags.VRM_MODEL_ALIAS or (p.model_name if p else "none")

    # ------------------------------------------------------------------ middleware
    def resolve_role(request: Request) -> Optional[str]:
        """Role of the caller: JWT access token -> its role; the static API token ->
        admin; nothing configured (development) -> admin; else None (401)."""
        token = os.environ.get("VRM_API_TOKEN", "")
        authz = request.headers.get("authorization", "")
        cred = authz[7:] if authz.startswith("Bearer ") else request.headers.get("x-api-key", "")
        if cred and ledger is not None and cred.startswith("sk-VRAM-"):
            info = ledger.verify(cred)
            if info is None:
                return None
            request.state.user = info["alias"]
            request.state.ledger_user = info
            return "user"
        if cred:
            claims = auth.access_claims(cred)
            if claims is not None:
                request.state.user = claims["sub"]
                return claims.get("role", "user")
            if token and hmac.compare_digest(cred, token):
                request.state.user = "api-token"
                return "admin"
        if not token and not auth.configured:
            request.state.user = "anonymous"
            return "admin"
        return None

    @app.middleware("http")
    async def protect(request: Request, call_next):
        path = request.url.path
        client = request.client.host if request.client else "?"
        origin = request.headers.get("origin")
        if not cors.allowed(origin):
            audit.log(client, request.method, path, 403, f"forbidden origin {origin}")
            return _err(403, "forbidden origin", "permission_error")
        if request.method == "OPTIONS" and origin:
            return Response(status_code=204, headers=cors.headers(origin))
        cl = request.headers.get("content-length")
        if cl and int(cl) > int(flags.VRM_MAX_BODY_BYTES):
            return _err(413, "request body too large")
        if path not in PUBLIC and path not in AUTH_OPEN:
            role = resolve_role(request)
            if role is None:
                audit.log(client, request.method, path, 401)
                return _err(401, "invalid or missing API token", "authentication_error")
            request.state.role = role
            need = required_role(request.method, path)
            if need and not role_allows(role, need):
                audit.log(client, request.method, path, 403, f"role {role} < {need}")
                return _err(403, f"role '{need}' required", "permission_error")
            secret = os.environ.get("VRM_HMAC_SECRET", "")
            if secret and request.method == "POST":
                body = await request.body()
                if not verify_signature(secret, request.method, path, body, request.headers.get("x-vrm-timestamp"),
                                        request.headers.get("x-vrm-signature")):
                    audit.log(client, request.method, path, 401, "bad signature")
                    return _err(401, "bad request signature", "authentication_error")
            if not flags.VRM_DISABLE_RATE_LIMIT and not limiter.allow(client):
                return _err(429, "rate limit exceeded", "rate_limit_error")
            if flags.VRM_READ_ONLY and path in ("/api/models/load", "/api/lora"):
                return _err(403, "server is read-only", "permission_error")
        resp = await call_next(request)
        if path not in PUBLIC:
            audit.log(client, request.method, path, resp.status_code)
        for k, v in cors.headers(origin).items():
            resp.headers[k] = v
        return resp

    def ledger_charge(request: Request, max_tokens: int):
        """402 response when a ledger user's balance is spent, else None after charging
        the request's max_tokens (a short balance is charged nothing and still served,
        as the reference does)."""
        info = getattr(request.state, "ledger_user", None)
        if info is None or ledger is None:
            return None
        bal = ledger.balance(info["id"])
        if bal is None or bal <= 0:
            return JSONResponse({"error": {"message": "Payment Required: insufficient VRAM credits",
                                           "type": "insufficient_credits"}, "credit_balance": bal or 0.0},
                                status_code=402)
        ledger.consume(info["id"], max_tokens)
        return None

    @app.post("/api/ledger/users")
    async def ledger_create_user(request: Request):
        if ledger is None:
            return _err(404, "no ledger configured (VRM_LEDGER_DB)", "not_found")
        body = await request.json()
        uid, key = ledger.create_user(str(body.get("alias", "user")), float(body.get("credits", 100.0)))
        return {"id": uid, "api_key": key, "credits": ledger.balance(uid)}

    @app.get("/api/ledger/balance")
    async def ledger_balance(request: Request):
        info = getattr(request.state, "ledger_user", None)
        if info is None or ledger is None:
            return _err(404, "not a ledger key", "not_found")
        return {"id": info["id"], "alias": info["alias"], "credit_balance": ledger.balance(info["id"])}

    # ------------------------------------------------------------------ accounts
    @app.post("/api/auth/login")
    async def auth_login(request: Request):
        body = await request.json()
        try:
            return auth.login(str(body.get("username", "")), str(body.get("password", "")))
        except AuthError as e:
            return _err(401, str(e), "authentication_error")

    @app.post("/api/auth/refresh")
    async def auth_refresh(request: Request):
        body = await request.json()
        try:
            return auth.refresh(str(body.get("refresh", "")))
        except (AuthError, ValueError) as e:
            return _err(401, str(e), "authentication_error")

    @app.get("/api/auth/me")
    async def auth_me(request: Request):
        return {"user": getattr(request.state, "user", None), "role": getattr(request.state, "role", None)}

    @app.post("/api/auth/change-password")
    async def auth_change_password(request: Request):
        body = await request.json()
        user = str(body.get("username") or getattr(request.state, "user", ""))
        if user != getattr(request.state, "user", None) and request.state.role != "admin":
            return _err(403, "only an admin changes another user's password", "permission_error")
        if not auth.change_password(user, str(body.get("old_password", "")), str(body.get("new_password", ""))):
            return _err(401, "invalid credentials", "authentication_error")
        return {"ok": True}

    @app.get("/api/auth/users")
    async def auth_list_users():
        return {"users": [{"username": u.username, "role": u.role} for u in auth.users.values()]}

    @app.post("/api/auth/users")
    async def auth_create_user(request: Request):
        body = await request.json()
        try:
            u = auth.create_user(str(body.get("username", "")), str(body.get("password", "")),
                                 str(body.get("role", "user")))
        except AuthError as e:
            return _err(400, str(e))
        return {"username": u.username, "role": u.role}

    # ------------------------------------------------------------------ helpers
    def run_guarded(fn, timeout: float):
        p = reg.pipeline
        if p is None or p.engine is None:
            return _err(503, "no model loaded", "service_unavailable")
        if not breaker.allow():
            METRICS.circuit_state.set(breaker.code())
            return _err(503, "circuit breaker open", "service_unavailable")
        if not queue.acquire():
            return _err(429, "queue full", "rate_limit_error")
        try:
            fut = executor.submit(fn, p)
            try:
                out = fut.result(timeout=timeout)
            except FutTimeout:
                breaker.failure()
                return _err(504, "generation timed out", "timeout")
            breaker.success()
            return out
        except ValidationError as e:
            return _err(400, str(e))
        except Exception as e:
            breaker.failure()
            METRICS.infer_errors.labels(type(e).__name__).inc()
            log.error("inference failed: %s", e)
            return _err(500, f"inference failed: {e}", "server_error")
        finally:
            queue.release()
            METRICS.circuit_state.set(breaker.code())

    def _finish_text(text: str, reason: Optional[str], stops) -> tuple:
        """Text cut before the first stop string (finish_reason "stop"), else as produced."""
        from ..pipeline import stop_index
        cut = stop_index(text, stops)
        if cut >= 0:
            return text[:cut], "stop"
        return text, ("stop" if reason in (None, "abort") else reason)

    def context_check(p, n_prompt: int, max_new: int):
        limit = p.engine.max_model_len
        if n_prompt + 1 > limit:
            raise ValidationError(f"context_length_exceeded: prompt has {n_prompt} tokens, limit {limit}")
        return min(max_new, limit - n_prompt)

    def sse(gen):
        def wrap():
            try:
                for chunk in gen:
                    yield f"data: {json.dumps(chunk)}\n\n"
            except Exception as e:
                yield f"data: {json.dumps({'error': {'message': str(e)}})}\n\n"
            yield "data: [DONE]\n\n"
        return StreamingResponse(wrap(), media_type="text/event-stream")

    # ------------------------------------------------------------------ inference
    async def _json(request: Request) -> Dict[str, Any]:
        try:
            return await request.json()
        except Exception:
            raise ValidationError("body must be JSON")

    @app.post("/v1/completions")
    @app.post("/api/generate")
    async def completions(request: Request):
        try:
            body = await _json(request)
            params = validate_generation_params(body)
        except ValidationError as e:
            return _err(400, str(e))
        prompt = body.get("prompt", "")
        if isinstance(prompt, list):
            prompt = prompt[0] if prompt and isinstance(prompt[0], str) else prompt
        METRICS.infer_requests.labels("completions").inc()
        p = reg.get(body.get("model") if body.get("model") not in (None, alias()) else None)
        if p is None:
            return _err(503, "no model loaded", "service_unavailable")
        try:
            n_prompt = len(p._encode(prompt))
            params["max_new_tokens"] = context_check(p, n_prompt, params["max_new_tokens"])
        except ValidationError as e:
            return _err(400, str(e), code="context_length_exceeded")
        denied = ledger_charge(request, params["max_new_tokens"] * int(params.get("n", 1) or 1))
        if denied is not None:
            return denied
        rid = f"cmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        stops, n_choices = params.pop("stop"), params.pop("n")
        if body.get("stream"):
            if n_choices > 1:
                return _err(400, "n > 1 is not supported with stream")

            def gen():
                for delta in p.generate_stream(prompt, stop=stops, **params):
                    yield {"id": rid, "object": "text_completion", "created": created, "model": alias(),
                           "choices": [{"index": 0, "text": delta, "finish_reason": None}]}
                yield {"id": rid, "object": "text_completion", "created": created, "model": alias(),
                       "choices": [{"index": 0, "text": "", "finish_reason": "stop"}]}
            return sse(gen())

        def work(pp):
            t0 = time.perf_counter()
            futs = [pp.submit(prompt, on_token=pp.stop_watcher(stops), **params) for _ in range(n_choices)]
            reqs = [f.result() for f in futs]
            choices = []
            for i, req in enumerate(reqs):
                text, finish = _finish_text(pp.tokenizer.decode(req.output_ids), req.finish_reason, stops)
                choices.append({"index": i, "text": text, "finish_reason": finish, "logprobs": None})
            dt = time.perf_counter() - t0
            n_out = sum(len(r.output_ids) for r in reqs)
            pp.history.record("completions", alias(), n_prompt, n_out, dt, reqs[0].ttft)
            return {"id": rid, "object": "text_completion", "created": created, "model": alias(),
                    "choices": choices,
                    "usage": {"prompt_tokens": n_prompt, "completion_tokens": n_out,
                              "total_tokens": n_prompt + n_out},
                    "timing": {"total_s": dt, "ttft_s": reqs[0].ttft, "tok_s": n_out / dt if dt > 0 else 0.0}}
        return await asyncio.get_running_loop().run_in_executor(
            None, lambda: run_guarded(work, float(flags.VRM_REQUEST_TIMEOUT)))

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        try:
            body = await _json(request)
            params = validate_generation_params(body)
            messages = body.get("messages")
            if not isinstance(messages, list) or not messages:
                raise ValidationError("messages must be a non-empty list")
        except ValidationError as e:
            return _err(400, str(e))
        METRICS.infer_requests.labels("chat").inc()
        p = reg.get(body.get("model") if body.get("model") not in (None, alias()) else None)
        if p is None:
            return _err(503, "no model loaded", "service_unavailable")
        prompt = build_chat_prompt(messages, body.get("tools"), body.get("tool_choice"))
        try:
            n_prompt = len(p._encode(prompt))
            params["max_new_tokens"] = context_check(p, n_prompt, params["max_new_tokens"])
        except ValidationError as e:
            return _err(400, str(e), code="context_length_exceeded")
        denied = ledger_charge(request, params["max_new_tokens"] * int(params.get("n", 1) or 1))
        if denied is not None:
            return denied
        rid = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        stops, n_choices = params.pop("stop"), params.pop("n")
        if body.get("stream"):
            if n_choices > 1:
                return _err(400, "n > 1 is not supported with stream")

            def gen():
                yield {"id": rid, "object": "chat.completion.chunk", "created": created, "model": alias(),
                       "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]}
                for delta in p.generate_stream(prompt, stop=stops, **params):
                    yield {"id": rid, "object": "chat.completion.chunk", "created": created, "model": alias(),
                           "choices": [{"index": 0, "delta": {"content": delta}, "finish_reason": None}]}
                yield {"id": rid, "object": "chat.completion.chunk", "created": created, "model": alias(),
                       "choices": [{"index": 0, "delta": {}, "finish_reason": "stop"}]}
            return sse(gen())

        def work(pp):
            t0 = time.perf_counter()
            futs = [pp.submit(prompt, on_token=pp.stop_watcher(stops), **params) for _ in range(n_choices)]
            reqs = [f.result() for f in futs]
            choices = []
            for i, req in enumerate(reqs):
                text, finish = _finish_text(pp.tokenizer.decode(req.output_ids), req.finish_reason, stops)
                msg, tool_finish = build_chat_message(text)
                choices.append({"index": i, "message": msg,
                                "finish_reason": "tool_calls" if tool_finish == "tool_calls" else finish})
            dt = time.perf_counter() - t0
            n_out = sum(len(r.output_ids) for r in reqs)
            pp.history.record("chat", alias(), n_prompt, n_out, dt, reqs[0].ttft)
            return {"id": rid, "object": "chat.completion", "created": created, "model": alias(),
                    "choices": choices,
                    "usage": {"prompt_tokens": n_prompt, "completion_tokens": n_out,
                              "total_tokens": n_prompt + n_out}}
        return await asyncio.get_running_loop().run_in_executor(
            None, lambda: run_guarded(work, float(flags.VRM_REQUEST_TIMEOUT)))

    @app.post("/v1/batch/completions")
    async def batch(request: Request):
        try:
            body = await _json(request)
            params = validate_generation_params(body)
            prompts = body.get("prompts")
            if not isinstance(prompts, list) or not prompts or len(prompts) > 32:
                raise ValidationError("prompts must be a list of 1..32 strings")
        except ValidationError as e:
            return _err(400, str(e))

        stops = params.pop("stop")
        params.pop("n")

        def work(pp):
            futs = [pp.submit(x, on_token=pp.stop_watcher(stops), **params) for x in prompts]
            reqs = [f.result() for f in futs]
            choices = []
            for i, r in enumerate(reqs):
                text, finish = _finish_text(pp.tokenizer.decode(r.output_ids), r.finish_reason, stops)
                choices.append({"index": i, "text": text, "finish_reason": finish})
            return {"object": "batch.completion", "model": alias(), "choices": choices}
        return await asyncio.get_running_loop().run_in_executor(
            None, lambda: run_guarded(work, float(flags.VRM_REQUEST_TIMEOUT)))

    @app.post("/api/infer")
    async def infer(request: Request):
        try:
            body = await _json(request)
            ids = body.get("input_ids")
            if ids is None:
                raise ValidationError("input_ids required")
        except ValidationError as e:
            return _err(400, str(e))
        topn = int(body.get("top", 20))

        def work(pp):
            lg = pp.infer(ids)
            v, i = lg.topk(min(topn, lg.numel()))
            out = {"argmax": int(lg.argmax()), "top": [[int(a), float(b)] for a, b in zip(i, v)]}
            if body.get("full"):
                out["logits"] = lg.tolist()
            return out
        return await asyncio.get_running_loop().run_in_executor(None, lambda: run_guarded(work, 60.0))

    # ------------------------------------------------------------------ models
    @app.get("/v1/models")
    @app.get("/api/models")
    def models():
        p = reg.pipeline
        data = []
        if p is not None:
            data.append({"id": alias(), "object": "model", "created": int(p.loaded_at or 0), "owned_by": "vramancer",
                         "mode": p.mode})
        return {"object": "list", "data": data}

    @app.post("/api/models/load")
    async def load_model(request: Request):
        body = await request.json()
        name = body.get("model")
        if not name:
            return _err(400, "model required")
        kw = {k: body[k] for k in ("num_gpus", "max_batch", "max_model_len", "kv_cache_dtype", "num_layers",
                                   "device") if k in body}
        loop = asyncio.get_running_loop()
        try:
            await loop.run_in_executor(None, lambda: reg.load(name, **kw))
        except Exception as e:
            return _err(500, f"load failed: {e}", "server_error")
        return {"status": "loaded", "model": name, "mode": reg.pipeline.mode}

    @app.get("/api/lora")
    def lora_list():
        p = reg.pipeline
        return p.lora.list_adapters() if p and p.lora else {"adapters": [], "active": None}

    @app.post("/api/lora")
    async def lora_op(request: Request):
        body = await request.json()
        p = reg.pipeline
        if p is None or p.lora is None:
            return _err(503, "no model loaded", "service_unavailable")
        op = body.get("op")
        try:
            if op == "load":
                n = p.lora.load_adapter(body["name"], body["path"])
                return {"loaded": body["name"], "projections": n}
            if op == "set":
                p.lora.set_adapter(body["name"])
            elif op == "disable":
                p.lora.disable()
            elif op == "delete":
                p.lora.delete_adapter(body["name"])
            else:
                return _err(400, "op must be load|set|disable|delete")
        except Exception as e:
            return _err(400, str(e))
        return p.lora.list_adapters()

    # ------------------------------------------------------------------ operations
    @app.get("/health")
    def health():
        p = reg.pipeline
        rep = {"status": "ok", "model_loaded": p is not None and p.engine is not None, "ts": time.time()}
        if p is not None and p.fault is not None:
            bad = [g for g, s in p.fault.status().items() if s["health"] not in ("healthy", "degraded")]
            if bad:
                rep["status"] = "degraded"
                rep["unhealthy_gpus"] = bad
        if p is not None and p.autoheal.scale < 1.0:
            rep["status"] = "degraded"
            rep["autoheal_scale"] = p.autoheal.scale
        return rep

    @app.get("/ready")
    def ready():
        p = reg.pipeline
        ok = p is not None and p.engine is not None and not reg.loading
        return JSONResponse({"ready": ok}, status_code=200 if ok else 503)

    @app.get("/live")
    def live():
        return {"live": True}

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse(METRICS.exposition().decode(), media_type="text/plain; version=0.0.4")

    @app.get("/api/status")
    @app.get("/api/pipeline/status")
    def status():
        p = reg.pipeline
        st = p.status() if p else {"loaded": False}
        st["startup_issues"] = app.state.startup_issues
        st["circuit_breaker"] = breaker.state
        return st

    @app.get("/api/gpu")
    @app.get("/api/gpu/info")
    def gpu():
        return {"gpus": monitor.poll()}

    @app.get("/api/system")
    def system():
        return health_report(monitor)

    @app.get("/api/queue/status")
    def queue_status():
        p = reg.pipeline
        return {"in_flight": queue.n, "limit": queue.limit,
                "waiting": len(p.engine.waiting) if p and p.engine else 0,
                "running": len(p.engine.running) if p and p.engine else 0}

    @app.get("/api/batcher/stats")
    def batcher_stats():
        p = reg.pipeline
        if p is None or p.engine is None:
            return {"enabled": False}
        d = dict(p.engine.stats)
        d.update(enabled=True, kv=p.engine.kv.stats(), speculative=p.engine.spec_stats.to_dict())
        return d

    @app.get("/api/history")
    def history(limit: int = 20):
        p = reg.pipeline
        return {"requests": p.history.recent(limit) if p else []}

    @app.get("/api/nodes")
    def nodes():
        from ..cluster.discovery import known_nodes
        return {"nodes": known_nodes()}

    # ------------------------------------------------------------------ cross-node workers
    from ..cluster import worker_api
    node = worker_api.NodeWorker()
    app.state.node_worker = node

    def _node_key(body) -> bytes:
        k = body.get("key") or os.environ.get("VRM_CLUSTER_KEY", "")
        return k.encode() if isinstance(k, str) else bytes(k)

    @app.get("/api/worker/model_info")
    def worker_model_info():
        return node.model_info()

    @app.post("/api/worker/load_partial")
    async def worker_load_partial(request: Request):
        try:
            body = await _json(request)
            info = await asyncio.get_running_loop().run_in_executor(None, lambda: node.load_partial(
                str(body["model"]), int(body.get("start_layer", 0)), int(body.get("end_layer", -1)),
                device=str(body.get("device", "cpu")), dtype=str(body.get("dtype", "float32")),
                seed=int(body.get("seed", 0)), tcp_port=body.get("tcp_port"),
                tcp_host=str(body.get("tcp_host", "127.0.0.1")), key=_node_key(body),
                num_pages=int(body.get("num_pages", 256))))
            return info
        except (KeyError, ValueError, ValidationError) as e:
            return _err(400, f"load_partial: {e}")

    @app.post("/api/worker/forward_layers")
    async def worker_forward_layers(request: Request):
        try:
            body = await _json(request)
            hidden = worker_api.decode_tensor(body["hidden"]) if body.get("hidden") else None
            ids = torch.as_tensor(body["input_ids"], dtype=torch.int32) if body.get("input_ids") is not None else None
            pos = torch.as_tensor(body["positions"], dtype=torch.int32) if body.get("positions") is not None else None
            out = await asyncio.get_running_loop().run_in_executor(
                None, lambda: node.forward_layers(hidden=hidden, input_ids=ids, positions=pos))
            kind = "logits" if node.end == node.cfg.num_layers else "hidden"
            return {"kind": kind, "layers": [node.start, node.end], "output": worker_api.encode_tensor(out)}
        except (KeyError, ValueError, ValidationError) as e:
            return _err(400, f"forward_layers: {e}")
        except RuntimeError as e:
            return _err(409, str(e))

    @app.post("/api/distributed/generate")
    async def distributed_generate(request: Request):
        try:
            body = await _json(request)
            prompts = body.get("prompts") or [body["prompt_ids"]]
            outs = await asyncio.get_running_loop().run_in_executor(None, lambda: worker_api.distributed_generate(
                str(body["model"]), [list(map(int, p)) for p in prompts], int(body.get("max_tokens", 16)),
                int(body["split"]), body.get("workers", []), device=str(body.get("device", "cpu")),
                dtype=str(body.get("dtype", "float32")), seed=int(body.get("seed", 0)), key=_node_key(body),
                num_pages=int(body.get("num_pages", 256)), temperature=float(body.get("temperature", 0.0))))
            return {"outputs": outs, "workers": len(body.get("workers", []))}
        except (KeyError, ValueError, ValidationError) as e:
            return _err(400, f"distributed generate: {e}")
        except (RuntimeError, OSError) as e:
            return _err(502, f"distributed generate: {e}", "server_error")

    @app.post("/api/swarm/awaken")
    async def swarm_awaken(request: Request):
        try:
            body = await _json(request)
            n = worker_api.wake_on_lan(body.get("macs", []), str(body.get("broadcast", "255.255.255.255")),
                                       int(body.get("port", 9)))
            return {"sent": n}
        except (ValueError, OSError, ValidationError) as e:
            return _err(400, f"awaken: {e}")

    @app.post("/api/benchmark")
    async def benchmark(request: Request):
        body = await request.json() if await request.body() else {}
        return await asyncio.get_running_loop().run_in_executor(
            None, lambda: run_guarded(lambda pp: pp.benchmark(int(body.get("prompt_len", 128)),
                                                              int(body.get("max_new_tokens", 32)),
                                                              int(body.get("batch", 1))), 600.0))

    @app.get("/")
    def root():
        return {"name": "VRAMancer-B200", "model": alias(), "docs": "/docs"}

    @app.get("/chat")
    def chat_page():
        return HTMLResponse(_CHAT_HTML)

    @app.get("/dashboard")
    def dashboard():
        return HTMLResponse(_DASHBOARD_HTML)

    return app


_CHAT_HTML = """<!doctype html><html><head><title>VRAMancer chat</title></head><body>
<h3>VRAMancer-B200</h3><div id=log style="white-space:pre-wrap;font-family:monospace"></div>
<input id=q size=80><button onclick="go()">send</button><script>
async function go(){const q=document.getElementById('q').value;const r=await fetch('/v1/chat/completions',{method:'POST',
headers:{'Content-Type':'application/json'},body:JSON.stringify({messages:[{role:'user',content:q}],max_tokens:128})});
const j=await r.json();document.getElementById('log').textContent+='> '+q+'\\n'+(j.choices?j.choices[0].message.content:JSON.stringify(j))+'\\n';}
</script></body></html>"""

_DASHBOARD_HTML = """<!doctype html><html><head><title>VRAMancer dashboard</title></head><body>
<h3>VRAMancer-B200 dashboard</h3><pre id=s></pre><script>
async function tick(){const a=await (await fetch('/api/gpu')).json();const b=await (await fetch('/api/batcher/stats')).json();
document.getElementById('s').textContent=JSON.stringify({gpus:a.gpus,batcher:b},null,1);}
setInterval(tick,2000);tick();</script></body></html>"""


def run_server(host: str = "0.0.0.0", port: int = 5030, pipeline=None, log_level: str = "info") -> None:
    import uvicorn
    app = create_app(pipeline)
    uvicorn.run(app, host=host, port=port, log_level=log_level)
