"""Tensor-parallel decode on 2, 4 or 8 GPUs (the most the box has) against the single-GPU engine on the same seeded weights, for both TP
engines: `tp.TPEngine` (op-by-op, NCCL all-reduces) and `tp.FusedTPEngine` (one persistent launch per token
and rank, the partials exchanged inside the kernel over NVLink).

Each rank runs the engine on its shard under a CUDA graph. Both engines are teacher-forced with the
single-GPU engine's greedy tokens, so they see the same inputs at every step. The checks:
* the layer-0 K/V rows the ranks append equal the TP=1 rows of their heads, bit for bit (layer 0 has no
  reduction before its qkv);
* the logits (each rank's vocabulary shard) are within 2e-2 rel-L2 of TP=1 at the first step and 5e-2 at
  every step (they differ only by the order of the fp32 partial sums after o_proj and down, amplified by the
  W8A8 re-quantisation of the next layer's input);
* every rank picks the same token at every step, and it is the TP=1 token at every step whose TP=1 top-2
  logit gap is more than twice the largest logit difference between the two runs at that step (a near-tie
  may legitimately flip under a different partial-sum order).

`test_fused_tp_recovers_after_a_peer_skips_a_step` covers the fused engine's failure handling without a GPU
fault: rank 1 stays alive, with its TP area mapped, but does not launch one step. Rank 0's kernel must give up
within its wait limit and report a timed-out exchange, and after `recover()` on both ranks the next step runs
clean on both. NVLS is off (NCCL_NVLS_ENABLE=0) and the kernel's exchange is plain peer stores and loads.
"""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 24
POS0 = 100


def _rendezvous(out_dir: str) -> str:
    """A file-based rendezvous in the test's own directory: no TCP port to pick, so no port a previous test's
    processes still hold can collide with it."""
    return "file://" + os.path.join(out_dir, "pg_rendezvous")


def _rank(rank, world, out_dir, fused):
    import datetime
    import torch.distributed as dist
    import model as M
    import tp as TP
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=_rendezvous(out_dir), rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    eng = None
    try:
        cfg = M.Config(layers=2, vocab=16384)
        dev = f"cuda:{rank}"
        m = TP.synthetic_shard(cfg, world, rank, max_seq=512, device=dev, seed=0)
        tokens = torch.load(os.path.join(out_dir, "tokens.pt"))
        eng = TP.FusedTPEngine(m) if fused else TP.TPEngine(m)
        eng.state.copy_(torch.tensor([POS0, 0], dtype=torch.int32))
        eng.token.fill_(int(tokens[0]))
        eng.capture()
        logits, got = [], []
        for i in range(STEPS):
            eng.token.fill_(int(tokens[i]))
            eng.graph.replay()
            logits.append(eng.logits.float().cpu())
            got.append(int(eng.token.item()))
        kv = (m.k_cache[0, 0, :, POS0].cpu(), m.v_cache[0, 0, :, POS0].cpu())
        err = eng.k.device_error()
        torch.save({"logits": torch.stack(logits), "tokens": got, "kv": kv, "vocab_offset": m.vocab_offset,
                    "device_error": err}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        if eng is not None:
            eng.release()
        dist.destroy_process_group()


WORLD = max([w for w in (2, 4, 8) if w <= torch.cuda.device_count()], default=0)


@pytest.mark.skipif(WORLD == 0, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [False, True], ids=["nccl", "fused"])
def test_tp2_matches_single_gpu(tmp_path, fused):
    import torch.multiprocessing as mp
    import model as M
    from generate import Engine
    cfg = M.Config(layers=2, vocab=16384)
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=512, device="cuda:0", seed=0)
    eng = Engine(m)
    eng.state.copy_(torch.tensor([POS0, 0], dtype=torch.int32))
    eng.token.fill_(1)
    eng.capture()
    tokens, logits = [1], []
    for i in range(STEPS):
        eng.token.fill_(tokens[i])
        eng.graph.replay()
        logits.append(eng.logits.float().cpu())
        tokens.append(int(eng.token.item()))
    kv = (m.k_cache[0, 0, :, POS0].cpu(), m.v_cache[0, 0, :, POS0].cpu())
    torch.save(torch.tensor(tokens), str(tmp_path / "tokens.pt"))
    del eng, m
    torch.cuda.empty_cache()
    mp.start_processes(_rank, args=(WORLD, str(tmp_path), fused), nprocs=WORLD,
                       start_method="spawn", join=True)
    ref = torch.stack(logits)
    full = torch.zeros_like(ref)
    rank_tokens = []
    for r in range(WORLD):
        d = torch.load(str(tmp_path / f"rank{r}.pt"))
        assert d["device_error"] == 0, d["device_error"]
        a, b = d["vocab_offset"], d["vocab_offset"] + d["logits"].shape[1]
        full[:, a:b] = d["logits"]
        per_step = [((d["logits"][i] - ref[i, a:b]).norm() / ref[i, a:b].norm()).item() for i in range(STEPS)]
        # the first step differs only through the fp32 partial-sum order of 2 layers; later steps also see
        # KV rows written with those differences, amplified by W8A8 re-quantisation
        assert per_step[0] < 2e-2 and max(per_step) < 5e-2, (r, per_step)
        kvr = 8 // WORLD
        heads = slice(kvr * r, kvr * r + kvr)
        assert torch.equal(d["kv"][0], kv[0][heads]) and torch.equal(d["kv"][1], kv[1][heads]), r
        rank_tokens.append(d["tokens"])
        print(f"rank {r}: logits rel-L2 first {per_step[0]:.4f} max {max(per_step):.4f}")
    assert all(t == rank_tokens[0] for t in rank_tokens), "ranks picked different tokens"
    got = rank_tokens[0]
    agree, unclear = 0, []
    for i in range(STEPS):
        top2 = torch.topk(ref[i], 2).values
        gap = float(top2[0] - top2[1])
        err = float((full[i] - ref[i]).abs().max())
        if got[i] == tokens[i + 1]:
            agree += 1
        elif gap > 2 * err:
            raise AssertionError(f"step {i}: TP={WORLD} token {got[i]} != TP=1 token {tokens[i + 1]} with a clear "
                                 f"top-2 gap {gap:.4f} > 2 x logit difference {err:.4f}")
        else:
            unclear.append((i, gap, err))
    print(f"TP={WORLD}: tokens agree {agree}/{STEPS}; near-tie flips {unclear}")


def _skip_rank(rank, world, out_dir):
    import datetime
    import time
    import torch.distributed as dist
    import model as M
    import tp as TP
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=_rendezvous(out_dir), rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    eng = None
    rec = {}
    try:
        cfg = M.Config(layers=2, vocab=16384)
        m = TP.synthetic_shard(cfg, world, rank, max_seq=512, device=f"cuda:{rank}", seed=0)
        eng = TP.FusedTPEngine(m)

        def run_step(pos, tok):
            eng.state.copy_(torch.tensor([pos, 0], dtype=torch.int32))
            eng.token.fill_(tok)
            eng.decode_step()
            torch.cuda.synchronize()

        run_step(POS0, 3)                       # a clean step on every rank
        rec["clean_error"] = eng.k.device_error()
        dist.barrier()
        if rank == 0:                           # the peers skip this step: rank 0's exchange waits must give up
            t0 = time.perf_counter()
            run_step(POS0 + 1, 5)
            rec["failed_step_s"] = time.perf_counter() - t0
            rec["failed_error"] = eng.k.device_error()
        dist.barrier()                          # the skipping ranks stay alive, areas mapped, until here
        eng.recover()
        run_step(POS0 + 1, 5)                   # every rank again, from the same state
        rec["after_error"] = eng.k.device_error()
        rec["after_token"] = int(eng.token.item())
        torch.save(rec, os.path.join(out_dir, f"skip{rank}.pt"))
    finally:
        if eng is not None:
            eng.release()
        dist.destroy_process_group()


@pytest.mark.skipif(WORLD == 0, reason="needs 2 GPUs")
def test_fused_tp_recovers_after_a_peer_skips_a_step(tmp_path, monkeypatch):
    import torch.multiprocessing as mp
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_skip_rank, args=(2, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    r0 = torch.load(str(tmp_path / "skip0.pt"))
    r1 = torch.load(str(tmp_path / "skip1.pt"))
    assert r0["clean_error"] == 0 and r1["clean_error"] == 0
    assert r0["failed_error"] & 4, r0          # DEVERR_GRID_TIMEOUT: a peer's partials never arrived
    assert r0["failed_step_s"] < 15.0, r0      # one wait limit (2 s), not one per wait
    assert r0["after_error"] == 0 and r1["after_error"] == 0, (r0, r1)
    assert r0["after_token"] == r1["after_token"]
    print(f"failed step gave up after {r0['failed_step_s']:.2f} s with error word {r0['failed_error']:#x}; "
          f"recovered, next token {r0['after_token']} on both ranks")
