"""The serving adapter (serve_adapter.py): `EngineModel.stream` and `pipelined`.

CPU: a list-backed fake torch and a fake engine check the bookkeeping a GPU run would otherwise be the first
to exercise: step 0 is the prefill's token and step s >= 1 reads out_tokens[s - 1] after decode replay s - 1;
exactly max_tokens - 1 replays run; at most `lookahead` steps are in flight; log-probs reach the host, the
first one taken before a graph capture's warm-up steps reuse the logits buffer; the prefill path follows
`chunk_min`; closing the stream early stops launching and drains; a device error raises.
GPU: the adapter over the real engine streams the same tokens as the engine run directly.
"""
from __future__ import annotations

import math
from contextlib import contextmanager
from types import SimpleNamespace

import pytest

import serve_adapter as SA


class FT:
    """A 1-D tensor over a Python list; slices share the list, like torch views."""

    def __init__(self, store, off=0, n=None):
        self.store, self.off = store, off
        self.n = len(store) - off if n is None else n

    def vals(self):
        return self.store[self.off:self.off + self.n]

    def __getitem__(self, k):
        if isinstance(k, slice):
            a, b, _ = k.indices(self.n)
            return FT(self.store, self.off + a, b - a)
        return self.store[self.off + k]

    def copy_(self, src, non_blocking=False):
        v = src.vals()
        assert len(v) == self.n
        self.store[self.off:self.off + self.n] = v
        return self

    def view(self, *shape):
        assert shape == (1,) and self.n == 1
        return self

    def float(self):
        return FT([float(x) for x in self.vals()])

    def max(self):
        return FT([max(self.vals())])

    def __sub__(self, o):
        return FT([a - b for a, b in zip(self.vals(), o.vals())])


class FakeTorch:
    int32, float32 = "int32", "float32"
    syncs = 0

    class cuda:
        class Stream:
            def wait_event(self, ev):
                assert ev.recorded

        class Event:
            recorded = False

            def record(self, stream=None):
                self.recorded = True

            def synchronize(self):
                assert self.recorded

        @staticmethod
        @contextmanager
        def stream(s):
            yield

        @staticmethod
        def synchronize():
            FakeTorch.syncs += 1

    @staticmethod
    def zeros(n, dtype=None, pin_memory=False, device=None):
        return FT([0] * n)

    @staticmethod
    def logsumexp(t, dim):
        return FT([math.log(sum(math.exp(x) for x in t.vals()))])

    @staticmethod
    def set_grad_enabled(flag):
        assert flag is False


V = 10


def logits_for(tok):
    row = [0.0] * V
    row[tok] = 2.0
    return row


LP = 2.0 - math.log(math.exp(2.0) + (V - 1))   # log-softmax of the argmax of logits_for()


class FakeEngine:
    """The engine interface the adapter uses: prefill / prefill_chunked, capture, graph.replay, out_tokens,
    logits, check."""

    def __init__(self, script, max_seq=64, error=0):
        self.script, self.max_seq, self.error = script, max_seq, error
        self.out_tokens = FT([-1] * max_seq)
        self.logits = FT([0.0] * V)
        self.m = SimpleNamespace(cfg=SimpleNamespace(vocab=V))
        self.graph = None
        self.replays = self.step = self.checks = 0
        self.path = None

    def _prefill(self, ids, path):
        self.path = path
        self.step = 0
        self.logits.copy_(FT(logits_for(self.script[0])))
        return FT([self.script[0]])

    def prefill(self, ids):
        return self._prefill(ids, "decode_graph")

    def prefill_chunked(self, ids):
        return self._prefill(ids, "chunked")

    def capture(self):
        self.logits.copy_(FT([9.0] * V))   # the warm-up steps overwrite the logits buffer
        self.graph = SimpleNamespace(replay=self._replay)

    def _replay(self):
        self.replays += 1
        tok = self.script[(self.step + 1) % len(self.script)]
        self.logits.copy_(FT(logits_for(tok)))
        self.out_tokens[self.step:self.step + 1].copy_(FT([tok]))
        self.step += 1

    def check(self):
        self.checks += 1
        if self.error:
            raise RuntimeError(f"decode step failed on the device (error word {self.error:#x})")


def adapter(script, lookahead=3, logprobs=True, chunk_min=16, **kw):
    eng = FakeEngine(script, **kw)
    em = SA.EngineModel.__new__(SA.EngineModel)
    em._setup(FakeTorch, eng, lookahead, logprobs, device="cpu", chunk_min=chunk_min)
    return em, eng


def test_stream_tokens_logprobs_and_replay_count():
    script = [5, 6, 7, 8, 9, 1, 3]
    em, eng = adapter(script)
    info = {}
    out = list(em.stream(list(range(20)), 6, True, info))
    assert [t for t, _ in out] == script[:6]
    # the first log-prob was taken before the capture's warm-up rewrote the logits
    assert all(abs(lp - LP) < 1e-9 for _, lp in out)
    assert eng.replays == 5 and eng.checks == 1
    assert info == {"prefill": "chunked"}


def test_prefill_path_follows_chunk_min():
    em, eng = adapter([4, 5], chunk_min=8)
    paths = []
    for P in (3, 7, 8, 30):
        info = {}
        list(em.stream([1] * P, 2, False, info))
        paths.append((info["prefill"], eng.path))
    assert paths == [("decode_graph",) * 2, ("decode_graph",) * 2, ("chunked",) * 2, ("chunked",) * 2]


def test_single_token_no_logprobs_needs_no_graph():
    em, eng = adapter([4, 5])
    assert list(em.stream([1, 2], 1, False, {})) == [(4, None)]
    assert eng.replays == 0 and eng.graph is None


def test_early_close_stops_launching_and_drains():
    em, eng = adapter(list(range(1, 9)), lookahead=3)
    before = FakeTorch.syncs
    g = em.stream([1, 2, 3], 40, False, {})
    assert [next(g)[0], next(g)[0]] == [1, 2]
    g.close()
    # steps 0..4 launched (2 collected + 3 in flight); step 0 is the prefill's, so 4 replays
    assert eng.replays == 4
    assert FakeTorch.syncs == before + 1 and eng.checks == 1


def test_device_error_raises_at_the_end_of_the_stream():
    em, eng = adapter([4, 5, 6], error=1)
    g = em.stream([1, 2], 3, False, {})
    assert [next(g)[0] for _ in range(3)] == [4, 5, 6]
    with pytest.raises(RuntimeError, match="error word 0x1"):
        next(g)


def test_size_checks():
    em, eng = adapter([4, 5])
    for ids, n in (([], 3), ([1], 0), ([1] * 60, 5)):
        with pytest.raises(ValueError, match="max_seq"):
            next(em.stream(ids, n, False, {}))


@pytest.mark.parametrize("lookahead", [1, 2, 5])
@pytest.mark.parametrize("n", [1, 3, 9])
def test_pipelined_order_and_depth(n, lookahead):
    events = []
    in_flight = set()

    def launch(i):
        events.append(("L", i))
        in_flight.add(i)
        assert len(in_flight) <= lookahead

    def collect(i):
        assert i in in_flight
        in_flight.discard(i)
        events.append(("C", i))
        return i

    assert list(SA.pipelined(n, lookahead, launch, collect)) == list(range(n))
    assert [i for k, i in events if k == "L"] == list(range(n))
    for i in range(n):   # step min(n - 1, i + lookahead - 1) was launched before step i was collected
        want = min(n - 1, i + lookahead - 1)
        assert events.index(("L", want)) < events.index(("C", i))


@pytest.mark.gpu
def test_stream_matches_the_engine_run_directly():
    import torch
    import model as M
    cfg = M.Config(layers=2, vocab=4096)
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=256, seed=5, norm_init="random")
    em = SA.EngineModel(m, lookahead=2, logprobs=True, fused=True, chunk_min=16)
    eng = em.engine
    for P in (24, 5):
        ids = [(i * 37 + 11) % cfg.vocab for i in range(P)]
        info = {}
        out = list(em.stream(ids, 10, True, info))
        assert info["prefill"] == ("chunked" if P >= 16 else "decode_graph")
        first = eng.prefill_chunked(ids) if P >= 16 else eng.prefill(ids)
        eng.step(9)
        want = [int(first)] + eng.out_tokens[:9].tolist()
        assert [t for t, _ in out] == want
        lps = [lp for _, lp in out]
        assert all(math.isfinite(lp) and lp <= 1e-6 for lp in lps)
        lf = eng.logits.float()
        assert abs(lps[-1] - float(lf.max() - torch.logsumexp(lf, 0))) < 1e-5
