"""HTTP serving front end over the continuous-batching scheduler (FastAPI; one engine, one scheduler thread).

Endpoints:

* ``POST /generate`` with ``{"input_ids": [...], "max_new_tokens": n, "stop": [...], "temperature": t,
  "top_k": k, "seed": s}`` returns ``{"output_ids": [...]}`` once the request finished; with ``"stream": true``
  the reply is a server-sent event stream: one ``data: {"token": t}`` event per generated token as the scheduler
  produces it, then ``data: {"output_ids": [...]}`` and ``data: [DONE]``;
* ``GET /metrics``: Prometheus text exposition of the engine's step metrics (tokens/s, TPOT percentiles);
* ``GET /health``.

Requests from many clients are queued into one ``Scheduler``; a single background thread steps it, so every
forward pass runs on one thread and concurrent requests share prefill and decode batches.  Token ids in, token ids
out (tokenisation belongs to the client).  Run with ``python -m carbon_b200.engine.server --preset small`` (one
GPU) or build ``make_app(engine)`` around an engine of your own.
"""
import argparse
import json
import os
import threading
from contextlib import asynccontextmanager
from typing import List

from .engine import Engine
from .scheduler import Scheduler


def make_app(engine: Engine, max_running: int = 256, prefill_tokens: int = 32768):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse
    from pydantic import BaseModel, Field

    class GenerateRequest(BaseModel):
        input_ids: List[int]
        max_new_tokens: int = Field(16, ge=1)
        stop: List[int] = []
        temperature: float = 0.0
        top_k: int = 0
        seed: int = 0
        stream: bool = False

    sched = Scheduler(engine, max_running=max_running, prefill_tokens=prefill_tokens)
    lock = threading.Condition()
    done = {}
    stop_flag = {"stop": False, "error": None}

    def loop():
        while True:
            with lock:
                while sched.idle() and not stop_flag["stop"]:
                    lock.wait(timeout=0.5)
                if stop_flag["stop"]:
                    return
                try:
                    sched.step()
                except Exception as e:          # a failed step fails every pending and later request
                    stop_flag["error"] = repr(e)
                    lock.notify_all()
                    return
                for jid, job in list(sched.finished.items()):
                    done[jid] = job.out
                    del sched.finished[jid]
                lock.notify_all()

    worker = threading.Thread(target=loop, name="carbon-scheduler", daemon=True)

    @asynccontextmanager
    async def lifespan(_app):
        worker.start()
        yield
        with lock:
            stop_flag["stop"] = True
            lock.notify_all()

    app = FastAPI(title="carbon-b200", lifespan=lifespan)

    @app.get("/health")
    def health():
        return {"status": "ok", "model": engine.cfg.n_layers}

    @app.post("/generate")
    def generate(req: GenerateRequest):
        if not req.input_ids or min(req.input_ids) < 0 or max(req.input_ids) >= engine.cfg.vocab_size:
            raise HTTPException(status_code=400, detail="input_ids must be non-empty token ids below vocab_size")
        with lock:
            if stop_flag["error"]:
                raise HTTPException(status_code=500, detail="engine failed: " + stop_flag["error"])
            try:
                jid = sched.submit(req.input_ids, req.max_new_tokens, tuple(req.stop), req.temperature, req.top_k,
                                   req.seed)
            except ValueError as e:                 # longer than the KV cache can ever hold
                raise HTTPException(status_code=400, detail=str(e))
            job = sched.jobs[jid]
            lock.notify_all()
            if req.stream:
                return StreamingResponse(_events(jid, job), media_type="text/event-stream")
            while jid not in done:
                if stop_flag["error"]:
                    raise HTTPException(status_code=500, detail="engine failed: " + stop_flag["error"])
                lock.wait(timeout=1.0)
            out = done.pop(jid)
        return {"output_ids": out}

    def _events(jid, job):
        sent = 0
        while True:
            with lock:
                while len(job.out) == sent and not job.done and not stop_flag["error"]:
                    lock.wait(timeout=1.0)
                if stop_flag["error"] and not job.done:
                    err = stop_flag["error"]
                    new, finished = [], None
                else:
                    err = None
                    new, finished = job.out[sent:], job.done
                    if finished:
                        done.pop(jid, None)
            if err is not None:
                yield "data: " + json.dumps({"error": "engine failed: " + err}) + "\n\n"
                return
            for t in new:
                yield "data: " + json.dumps({"token": t}) + "\n\n"
            sent += len(new)
            if finished:
                yield "data: " + json.dumps({"output_ids": list(job.out)}) + "\n\n"
                yield "data: [DONE]\n\n"
                return

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        with lock:
            return engine.metrics.prometheus()

    return app


def main():
    from ..config import PRESETS
    from ..models.weights import WeightSource

    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="small", choices=sorted(PRESETS))
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--pages", type=int, default=2048)
    ap.add_argument("--checkpoint", default=None)
    a = ap.parse_args()
    cfg = PRESETS[a.preset]()
    if a.checkpoint and os.path.exists(os.path.join(a.checkpoint, "config.json")):
        from ..config import ModelConfig

        cfg = ModelConfig.from_hf(a.checkpoint)           # a Hugging Face DeepSeek checkpoint directory
    if a.checkpoint:
        from ..models.checkpoint import CheckpointSource

        src = CheckpointSource(cfg, a.checkpoint)
    else:
        src = WeightSource(cfg, seed=0)
    eng = Engine(cfg, device=a.device, source=src, num_pages=a.pages, page_size=64, cuda_graphs=a.device != "cpu")
    import uvicorn

    uvicorn.run(make_app(eng), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
