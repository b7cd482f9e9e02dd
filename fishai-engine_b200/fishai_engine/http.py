"""HTTP front end of the token loop on the device model: the reference's
model routes (src/http.rs:839-853) with its request/response shapes and
validation rules, served by FastAPI (uvicorn) instead of axum.

  GET  /health                   src/http.rs:391-399
  POST /api/sample               src/http.rs:401-475  (Sampler::sample on the device)
  POST /api/model/load           src/http.rs:603-695  (allowed-directory check, src/http.rs:570-600)
  POST /api/model/generate       src/http.rs:697-766
  GET  /api/model/status         src/http.rs:768-790
  POST /api/model/generate/stream   NEW: not in the reference, which answers
                                    /api/model/generate with one JSON body.  The
                                    same generation as Server-Sent Events, one
                                    event per generated token, then a final
                                    event with the counts.

As in the reference, the prompt text maps to token ids by Unicode code point
and ids map back to text the same way (src/http.rs:745-756); the reference
does not wire its BpeTokenizer into this route.  Categorical draws use the
device's Philox stream keyed by the request's optional `seed` (default 0)
where the reference draws from an unseeded generator.  The chat, prompt,
memory, thinking and security routes (auth, rate limits) are not part of the
token path and are not served here.

  python -m fishai_engine.http --host 127.0.0.1 --port 8080 --model-dir /models
"""
import json
import os
import threading
from typing import List, Optional

VERSION = "0.2.0"


def _sanitize_text(ids: List[int]) -> str:
    out = []
    for i in ids:
        try:
            out.append(chr(i))
        except (ValueError, OverflowError):
            out.append("�")
    return "".join(out)


def validate_model_path(path: str, allowed_dirs: List[str]) -> str:
    """src/http.rs:570-600: the canonical path must lie inside one of the
    allowed directories (none configured: any path)."""
    if not os.path.exists(path):
        raise PermissionError(f"model file does not exist: {path}")
    canonical = os.path.realpath(path)
    if not allowed_dirs:
        return canonical
    for d in allowed_dirs:
        cd = os.path.realpath(d)
        if os.path.commonpath([canonical, cd]) == cd:
            return canonical
    raise PermissionError(f"path '{path}' is not inside the allowed model directories: {allowed_dirs}")


def create_app(model_dirs: Optional[List[str]] = None, device: int = 0, max_text_length: int = 32768,
               max_logits_length: int = 1_000_000, max_generate_tokens: int = 4096, use_tc_prefill: bool = False):
    """The FastAPI application.  One model at a time, generations serialised
    (the device model is one stream)."""
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, StreamingResponse

    app = FastAPI(title="fishai-engine (B200)", version=VERSION)
    state = {"model": None, "info": None}
    lock = threading.Lock()

    def err(status, msg):
        return JSONResponse(status_code=status, content={"error": msg, "code": status})

    @app.get("/health")
    def health():
        return {"status": "ok", "version": VERSION, "engine": "fishai-engine (B200 CUDA)",
                "model_loaded": state["model"] is not None}

    @app.post("/api/sample")
    async def sample(request: Request):
        from .sampling import Sampler, SamplerConfig

        body = await request.json()
        logits = body.get("logits") or []
        if not logits:
            return err(400, "logits must not be empty")
        if len(logits) > max_logits_length:
            return err(400, f"logits longer than the limit ({max_logits_length})")
        cfg = SamplerConfig()
        o = body.get("config") or {}
        if o.get("temperature") is not None:
            t = float(o["temperature"])
            if not 0.0 <= t <= 2.0:
                return err(400, "temperature must be within 0.0..2.0")
            cfg.temperature = t
        if o.get("top_k") is not None:
            cfg.top_k = int(o["top_k"])
        if o.get("top_p") is not None:
            p = float(o["top_p"])
            if not 0.0 <= p <= 1.0:
                return err(400, "top_p must be within 0.0..1.0")
            cfg.top_p = p
        if o.get("repetition_penalty") is not None:
            r = float(o["repetition_penalty"])
            if r <= 0.0:
                return err(400, "repetition_penalty must be > 0")
            cfg.repetition_penalty = r
        if o.get("frequency_penalty") is not None:
            cfg.frequency_penalty = float(o["frequency_penalty"])
        if o.get("presence_penalty") is not None:
            cfg.presence_penalty = float(o["presence_penalty"])
        s = Sampler(cfg, len(logits), seed=int(body.get("seed", 0)))
        for tok, count in enumerate(body.get("token_freq") or []):
            for _ in range(int(count)):
                s.observe_token(tok)
        for tok, present in enumerate(body.get("token_present") or []):
            if present:
                s.observe_token(tok)
        with lock:
            token = s.sample(logits)
        return {"token_id": int(token)}

    def model_info(cfg):
        return {"n_layers": cfg.n_layers, "n_heads": cfg.n_heads, "n_kv_heads": cfg.n_kv_heads,
                "head_dim": cfg.head_dim, "n_embd": cfg.n_embd, "vocab_size": cfg.vocab_size,
                "context_len": cfg.context_len, "n_ff": cfg.n_ff}

    @app.post("/api/model/load")
    async def load(request: Request):
        from ._lib import FishaiError
        from .model import ModelWeights

        body = await request.json()
        try:
            path = validate_model_path(str(body.get("path", "")), model_dirs or [])
        except PermissionError as e:
            return JSONResponse(status_code=403, content={"success": False, "message": str(e)})
        try:
            with lock:
                if state["model"] is not None:
                    state["model"].close()
                    state["model"] = None
                m = ModelWeights.load_from_gguf(path, device=device, use_tc_prefill=use_tc_prefill)
                state["model"], state["info"] = m, model_info(m.config)
        except FishaiError as e:
            return JSONResponse(status_code=400, content={"success": False, "message": f"cannot load model: {e}"})
        c = m.config
        return {"success": True, "config": state["info"],
                "message": f"model loaded: {c.n_layers} layers, {c.n_heads} heads, {c.n_embd} dims, "
                           f"{c.vocab_size} vocab"}

    @app.get("/api/model/status")
    def status():
        return {"loaded": state["model"] is not None, "config": state["info"]}

    def gen_config(body):
        from .model import GenerationConfig

        prompt = str(body.get("prompt", ""))
        ids = [ord(ch) for ch in prompt]
        # max_tokens counts the prompt, as GenerationState does (src/model.rs:683-686)
        cfg = GenerationConfig(max_tokens=min(int(body.get("max_tokens") or 256), max_generate_tokens),
                               temperature=min(max(float(body.get("temperature", 0.7) or 0.0), 0.0), 2.0),
                               top_k=int(body.get("top_k", 40)),
                               top_p=min(max(float(body.get("top_p", 0.95)), 0.0), 1.0),
                               repetition_penalty=float(body.get("repetition_penalty", 1.15)))
        return prompt, ids, cfg, int(body.get("seed", 0))

    def check_request(prompt, ids):
        m = state["model"]
        if len(prompt) > max_text_length:
            return err(400, f"prompt too long (max {max_text_length} characters)")
        if m is None:
            return JSONResponse(status_code=503, content={
                "success": False, "message": "no model loaded: POST /api/model/load first"})
        if not ids:
            return err(400, "prompt must not be empty")
        V = m.config.vocab_size
        if any(i >= V for i in ids):
            return err(400, f"prompt has characters whose code point is outside the vocabulary ({V})")
        return None

    @app.post("/api/model/generate")
    async def generate(request: Request):
        from .model import GenerationState

        prompt, ids, cfg, seed = gen_config(await request.json())
        bad = check_request(prompt, ids)
        if bad is not None:
            return bad
        with lock:
            out = GenerationState(state["model"], cfg, seed=seed).generate(ids)
        return {"success": True, "text": _sanitize_text(out), "token_ids": out, "n_prompt_tokens": len(ids),
                "n_generated_tokens": len(out), "message": None}

    @app.post("/api/model/generate/stream")
    async def generate_stream(request: Request):
        from .kv_cache import KVCache
        from .model import GenerationState

        prompt, ids, cfg, seed = gen_config(await request.json())
        bad = check_request(prompt, ids)
        if bad is not None:
            return bad

        def events():
            with lock:
                m = state["model"]
                st = GenerationState(m, cfg, seed=seed)
                st.kv_cache = KVCache(m, max(cfg.max_tokens + 1, 16), 1, st.kv_dtype)
                m.prefill(ids, 0, st.kv_cache, want_logits=False)
                st.token_ids, st.pos = list(ids), len(ids)
                tok, n = ids[-1], 0
                while True:
                    nxt = st.generate_step(tok)
                    if nxt is None:
                        break
                    n += 1
                    yield f"data: {json.dumps({'token_id': nxt, 'text': _sanitize_text([nxt])})}\n\n"
                    tok = nxt
                yield f"data: {json.dumps({'done': True, 'n_prompt_tokens': len(ids), 'n_generated_tokens': n})}\n\n"

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.exception_handler(404)
    async def not_found(request, exc):
        return err(404, f"not found: {request.url.path}")

    return app


def main():
    import argparse

    import uvicorn

    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--model-dir", action="append", default=[])
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--tc-prefill", action="store_true")
    a = ap.parse_args()
    uvicorn.run(create_app(a.model_dir, a.device, use_tc_prefill=a.tc_prefill), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
