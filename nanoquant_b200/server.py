"""OpenAI-compatible serving of a packed NanoQuant Llama checkpoint on the B200 kernels.

Mirrors the reference's src/nanoquant/openai_server.py (:168-404): the same endpoints
(``GET /health``, ``GET /v1/models``, ``POST /v1/chat/completions``), the same bearer-token check
on every endpoint, the same request validation and error messages (no streaming, n == 1,
max_tokens bounds, no custom stop strings, temperature / top_p / top_k ranges), one request at a
time, and the same response body (chat.completion with usage counts).  What differs:

* the model is this package's decoder (nanoquant_b200.decoder.Decoder) loaded from the packed
  checkpoint with no dense unpack (nanoquant_b200.loader), running greedy decoding through its
  captured CUDA graph (temperature 0) or sampling from its logits (temperature > 0, top-k / top-p);
* the architecture is Llama (what the decoder implements); the reference's Qwen tool-call parsing
  is not applied (tool definitions are passed to the chat template when the tokenizer has one).

    python -m nanoquant_b200.server --checkpoint ckpt.pt --model-id <local HF model dir> --api-key KEY
"""
import argparse
import hmac
import logging
import threading
import time
import uuid
from typing import Any, List, Optional

import torch

LOGGER = logging.getLogger("nanoquant_b200.server")


class DecoderEngine:
    """Generation with one batch-1 decoder: greedy through the captured decode graph, sampled
    from the step logits otherwise; stops at ``eos_token_id`` or after ``max_new_tokens``."""

    def __init__(self, dec, eos_token_id: Optional[int] = None):
        self.dec = dec
        self.eos = eos_token_id
        self.graph = dec.capture(warmup=1)
        self.host_in = torch.empty(1, dtype=torch.long).pin_memory()
        self.host_out = torch.empty(1, dtype=torch.long).pin_memory()

    @property
    def max_seq(self) -> int:
        return self.dec.max_seq

    @torch.no_grad()
    def generate(self, input_ids: List[int], max_new_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                 top_k: int = 0, seed: Optional[int] = None) -> List[int]:
        dec = self.dec
        if len(input_ids) + max_new_tokens >= dec.max_seq:
            raise ValueError(f"prompt ({len(input_ids)}) + max_tokens ({max_new_tokens}) exceed the context "
                             f"of {dec.max_seq - 1} tokens")
        gen = None
        if seed is not None:
            gen = torch.Generator(device=dec.device)
            gen.manual_seed(int(seed))
        first = int(dec.prefill(torch.tensor(input_ids, dtype=torch.long, device=dec.device))[0])
        if temperature > 0:  # the prefill's token is greedy: redo it from the last position's logits
            dec.pos.sub_(1)
            dec.seq_len.sub_(1)
            dec.tokens.fill_(int(input_ids[-1]))
            first = None
        out: List[int] = []
        tok = first
        while len(out) < max_new_tokens:
            if temperature > 0:
                logits = dec.step_logits().float()[0] / temperature
                tok = sample(logits, top_p, top_k, gen)
                dec.tokens.fill_(tok)
                dec.pos.add_(1)
                dec.seq_len.add_(1)
            elif out:  # greedy: the graphed step (host token id in, next id out)
                self.host_in.fill_(tok)
                tok = int(self.graph.generate(self.host_in, self.host_out)[0])
            out.append(tok)
            if self.eos is not None and tok == self.eos:
                break
        return out


def sample(logits: torch.Tensor, top_p: float, top_k: int, gen=None) -> int:
    """One token from temperature-scaled logits with top-k then nucleus (top-p) filtering."""
    if top_k > 0:
        kth = torch.topk(logits, min(top_k, logits.numel())).values[-1]
        logits = torch.where(logits < kth, torch.full_like(logits, float("-inf")), logits)
    probs = torch.softmax(logits, dim=-1)
    if 0 < top_p < 1:
        sp, idx = torch.sort(probs, descending=True)
        keep = torch.cumsum(sp, 0) - sp < top_p
        sp = torch.where(keep, sp, torch.zeros_like(sp))
        probs = torch.zeros_like(probs).scatter_(0, idx, sp)
    return int(torch.multinomial(probs / probs.sum(), 1, generator=gen)[0])


def _require_api_key(request, api_key: str) -> None:
    from fastapi import HTTPException
    supplied = request.headers.get("authorization", "")
    supplied = supplied[7:].strip() if supplied.lower().startswith("bearer ") else ""
    if not hmac.compare_digest(supplied, api_key):
        raise HTTPException(status_code=401, detail="Invalid or missing bearer token.")


def _messages(raw: Any) -> List[dict]:
    from fastapi import HTTPException
    if not isinstance(raw, list) or not raw:
        raise HTTPException(status_code=400, detail="messages must be a non-empty array.")
    out = []
    for m in raw:
        if not isinstance(m, dict) or "role" not in m:
            raise HTTPException(status_code=400, detail="every message needs a role.")
        content = m.get("content", "")
        if isinstance(content, list):  # OpenAI content parts: keep the text parts
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        out.append({"role": str(m["role"]), "content": "" if content is None else str(content)})
    return out


def create_app(args: argparse.Namespace, engine=None, tokenizer=None):
    """The FastAPI app.  ``engine`` / ``tokenizer`` are built from ``args`` when not given."""
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse

    if not args.api_key:
        raise ValueError("Pass a random --api-key; the OpenAI endpoint is bearer-token protected.")
    started = time.monotonic()
    if tokenizer is None:
        from transformers import AutoTokenizer
        tokenizer = AutoTokenizer.from_pretrained(args.model_id, revision=args.revision)
    if engine is None:
        if not torch.cuda.is_available():
            raise RuntimeError("NanoQuant inference requires a CUDA GPU.")
        from transformers import AutoConfig

        from .loader import load_compressed_decoder
        dtype = torch.bfloat16 if args.dtype == "bfloat16" else torch.float16
        conf = AutoConfig.from_pretrained(args.model_id, revision=args.revision)
        max_seq = args.seqlen if args.seqlen > 0 else int(getattr(conf, "max_position_embeddings", 4096))
        dec = load_compressed_decoder(conf, args.checkpoint, max_seq=max_seq, dtype=dtype, device=args.device)
        engine = DecoderEngine(dec, eos_token_id=tokenizer.eos_token_id)
    app = FastAPI(title="NanoQuant OpenAI-compatible API (B200 kernels)", version="1.0.0")
    lock = threading.Lock()
    app.state.ready_info = {"model": args.model_name, "kernel": "b200", "device": args.device, "dtype": args.dtype,
                            "startup_seconds": round(time.monotonic() - started, 3), "max_tokens": args.max_tokens}

    @app.get("/health")
    def health(request: Request):
        _require_api_key(request, args.api_key)
        return {"status": "ok", **app.state.ready_info}

    @app.get("/v1/models")
    def models(request: Request):
        _require_api_key(request, args.api_key)
        return {"object": "list", "data": [{"id": args.model_name, "object": "model", "owned_by": "nanoquant"}]}

    @app.post("/v1/chat/completions")
    def chat_completions(request: Request, payload: dict):
        _require_api_key(request, args.api_key)
        if payload.get("stream"):
            raise HTTPException(status_code=400, detail="Streaming responses are not enabled in this server.")
        if int(payload.get("n", 1)) != 1:
            raise HTTPException(status_code=400, detail="Only n=1 is supported.")
        messages = _messages(payload.get("messages"))
        tools = payload.get("tools") or []
        if not isinstance(tools, list):
            raise HTTPException(status_code=400, detail="tools must be an array.")
        kwargs = {"tools": tools} if tools and payload.get("tool_choice", "auto") != "none" else {}
        try:
            ids = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=True, **kwargs)
            if isinstance(ids, dict):
                ids = ids["input_ids"]
            if hasattr(ids, "tolist"):
                ids = ids.tolist()
            if ids and isinstance(ids[0], list):
                ids = ids[0]
        except Exception as error:
            raise HTTPException(status_code=400, detail=f"Could not format messages/tools: {error}") from error
        max_new = int(payload.get("max_completion_tokens", payload.get("max_tokens", args.max_tokens)))
        if max_new < 1 or max_new > args.max_tokens:
            raise HTTPException(status_code=400,
                                detail=f"max_tokens must be between 1 and {args.max_tokens} for this server.")
        if payload.get("stop") not in (None, [], ""):
            raise HTTPException(status_code=400,
                                detail="Custom stop strings are not supported; use the model EOS token.")
        temperature = float(payload.get("temperature", 1.0))
        top_p = float(payload.get("top_p", 0.95))
        top_k = int(payload.get("top_k", 20))
        if temperature < 0 or not 0 < top_p <= 1 or top_k < 1:
            raise HTTPException(status_code=400, detail="temperature must be non-negative and top_p in (0, 1].")
        try:
            with lock, torch.inference_mode():
                completion = engine.generate(ids, max_new, temperature, top_p, top_k, payload.get("seed"))
        except ValueError as error:
            raise HTTPException(status_code=400, detail=str(error)) from error
        except Exception as error:
            LOGGER.exception("NanoQuant generation failed")
            raise HTTPException(status_code=500, detail=f"Generation failed: {type(error).__name__}: {error}") from error
        text = tokenizer.decode(completion, skip_special_tokens=False)
        finish = "length" if len(completion) >= max_new else "stop"
        return JSONResponse({
            "id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion", "created": int(time.time()),
            "model": args.model_name,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": finish}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": len(completion),
                      "total_tokens": len(ids) + len(completion)}})

    return app


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--checkpoint", required=True, help="packed NanoQuant checkpoint (file or directory)")
    p.add_argument("--model-id", required=True, help="local HF model directory (config + tokenizer)")
    p.add_argument("--model-name", default="nanoquant-b200", help="ID returned by /v1/models")
    p.add_argument("--revision", default=None)
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--dtype", choices=("bfloat16", "float16"), default="float16")
    p.add_argument("--seqlen", type=int, default=-1)
    p.add_argument("--max-tokens", type=int, default=8192)
    p.add_argument("--api-key", required=True, help="bearer token required on every API endpoint")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--log-level", choices=("debug", "info", "warning", "error"), default="info")
    return p.parse_args(argv)


def main() -> None:
    import uvicorn
    args = parse_args()
    logging.basicConfig(level=getattr(logging, args.log_level.upper()), format="%(asctime)s %(levelname)s %(message)s")
    uvicorn.run(create_app(args), host=args.host, port=args.port, log_level=args.log_level)


if __name__ == "__main__":
    main()
