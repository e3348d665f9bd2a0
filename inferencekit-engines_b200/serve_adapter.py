"""Serving adapter: the B200 engine as a token stream for a request server.

Mirrors the reference's real-engine adapter, `EngineModel` (qwen3-8b-fp8_rtx-5090/serve.py:878-1019), and its
`pipelined` helper (serve.py:812-826): the interface a FIFO, one-request-at-a-time server drives.

* `stream(prompt_ids, max_tokens, logprobs, info)` yields `(token, logprob or None)` for up to max_tokens
  steps; a server that meets a stop token closes the generator.
* Step 0 is the prefill's token. Step s >= 1 is decode-graph replay s - 1, which writes `out_tokens[s - 1]`.
* Up to `lookahead` steps are launched ahead of the one being collected. Each step's token (and log-prob) is
  copied device -> pinned host on a side stream, behind an event recorded after the step, so the host waits
  only for the copy of the step it yields while the GPU already runs the next ones.
* Closing the generator stops launching; the steps in flight finish (one device sync) before the next request,
  and the engine's device error word is read, so a step that gave up on the device raises instead of
  streaming garbage.

Differences from the reference: prompts of at least `chunk_min` tokens are prefilled by
`Engine.prefill_chunked` (the batched forward), shorter ones position by position through the decode graph
(`Engine.prefill`); `info["prefill"]` names the path. The reference's per-length prefill graphs have no
counterpart here. Log-probs are the log-softmax of the chosen (argmax) token over the step's bf16 logits,
computed on the device, as the reference does.
"""
from __future__ import annotations


def pipelined(n: int, lookahead: int, launch, collect):
    """Yield collect(0), ..., collect(n - 1) in order, keeping up to `lookahead` steps launched ahead of the
    one being collected: step i + lookahead is launched before step i's result is yielded. launch(i) only
    enqueues work; collect(i) blocks until step i's result is on the host. Closing the generator launches
    nothing more."""
    ahead = max(1, int(lookahead))
    next_launch = 0
    for i in range(n):
        while next_launch < n and next_launch < i + ahead:
            launch(next_launch)
            next_launch += 1
        result = collect(i)
        if next_launch < n:
            launch(next_launch)
            next_launch += 1
        yield result


class EngineModel:
    """generate.Engine behind the serving interface. `EngineModel(model)` builds the engine (fused step by
    default), captures its decode graph and warms the chunked prefill once."""

    def __init__(self, model, lookahead: int = 2, logprobs: bool = True, fused: bool = True, chunk_min: int = 16,
                 warmup: bool = True):
        import torch
        from generate import Engine
        eng = Engine(model, fused=fused)
        self._setup(torch, eng, lookahead, logprobs, chunk_min=chunk_min)
        if warmup:
            with torch.no_grad():
                ids = [(i * 7919 + 13) % model.cfg.vocab for i in range(max(chunk_min, 2))]
                list(self.stream(ids, 2, logprobs, {}))                        # chunked prefill + graph capture
                list(self.stream(ids[: max(1, min(chunk_min - 1, 4))], 2, logprobs, {}))   # decode-path prefill

    def _setup(self, torch, eng, lookahead, logprobs, device="cuda", chunk_min: int = 16):
        """Streaming buffers (tests call this with a fake torch and a fake engine)."""
        self.torch, self.engine = torch, eng
        self.max_seq = eng.max_seq
        self.vocab_size = eng.m.cfg.vocab
        self.lookahead = max(1, int(lookahead))
        self.logprobs_supported = bool(logprobs)
        self.chunk_min = int(chunk_min)
        self.copy_stream = torch.cuda.Stream()
        self.host_tok = torch.zeros(self.max_seq, dtype=torch.int32, pin_memory=True)
        self.host_lp = torch.zeros(self.max_seq, dtype=torch.float32, pin_memory=True)
        self.lp_dev = torch.zeros(self.max_seq, dtype=torch.float32, device=device)
        # an event is re-recorded only after its step was collected: more slots than steps in flight
        ring = self.lookahead + 2
        self.ev_step = [torch.cuda.Event() for _ in range(ring)]
        self.ev_copied = [torch.cuda.Event() for _ in range(ring)]

    def describe(self) -> dict:
        """What a server reports about the engine (its /config)."""
        eng = self.engine
        return {"engine": "b200-qwen3-fp8", "fused_step": bool(getattr(eng, "fused", False)),
                "decode_graph": getattr(eng, "graph", None) is not None, "max_context": self.max_seq,
                "vocab_size": self.vocab_size, "lookahead": self.lookahead, "logprobs": self.logprobs_supported,
                "prefill": f"chunked (tcgen05 batched linear) for >= {self.chunk_min} tokens, else the decode graph",
                "batch": 1, "scheduling": "FIFO, one request at a time", "sampling": "greedy"}

    def _logprob_into(self, s):
        """lp_dev[s] = log-softmax of the argmax of the engine's current logits (on the device)."""
        lf = self.engine.logits.float()
        self.lp_dev[s:s + 1].copy_((lf.max() - self.torch.logsumexp(lf, 0)).view(1))
        return self.lp_dev[s:s + 1]

    def stream(self, prompt_ids, max_tokens, logprobs, info):
        torch, eng = self.torch, self.engine
        torch.set_grad_enabled(False)   # thread-local: this runs on the server's worker thread
        P = len(prompt_ids)
        if P < 1 or max_tokens < 1 or P + max_tokens > self.max_seq:
            raise ValueError(f"prompt of {P} tokens + {max_tokens} new tokens does not fit max_seq {self.max_seq}")
        chunked = P >= self.chunk_min and getattr(getattr(eng, "m", None), "kv_dtype", "bf16") == "bf16"
        first = eng.prefill_chunked(prompt_ids) if chunked else eng.prefill(prompt_ids)   # device tensor, no sync
        info["prefill"] = "chunked" if chunked else "decode_graph"
        want_lp = bool(logprobs) and self.logprobs_supported
        first_lp = self._logprob_into(0) if want_lp else None   # before a capture's warm-up steps reuse the logits
        if eng.graph is None and max_tokens > 1:
            eng.capture()   # first request only: the state after a prefill is a valid one to capture from
        R = len(self.ev_step)

        def launch(s):
            if s == 0:
                src, lp_src = first.view(1), first_lp
            else:
                eng.graph.replay()
                src = eng.out_tokens[s - 1:s]
                lp_src = self._logprob_into(s) if want_lp else None
            ev = self.ev_step[s % R]
            ev.record()
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(ev)
                self.host_tok[s:s + 1].copy_(src, non_blocking=True)
                if lp_src is not None:
                    self.host_lp[s:s + 1].copy_(lp_src, non_blocking=True)
                self.ev_copied[s % R].record(self.copy_stream)

        def collect(s):
            self.ev_copied[s % R].synchronize()
            return int(self.host_tok[s]), (float(self.host_lp[s]) if want_lp else None)

        try:
            yield from pipelined(max_tokens, self.lookahead, launch, collect)
        finally:
            torch.cuda.synchronize()   # steps still in flight (after a stop token) end before the next request
            del first
            eng.check()
