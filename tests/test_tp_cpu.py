"""Tensor-parallel host logic on CPU: the shards of `tp.py` tile every full matrix exactly, and a gloo
world_size-2 run of the oracle layer on those shards (with the all-reduces the TP engine issues) equals the
unsharded oracle layer, including the vocab-parallel argmax."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import model as M
import tp as TP
from oracle import qwen3_ref as O

SEED = 7


def small_cfg(vocab=1024):
    return M.Config(layers=1, vocab=vocab)


@pytest.mark.parametrize("tp", [2, 8])
@pytest.mark.parametrize("scale_mode", ["channel", "block"])
def test_shards_tile_the_full_matrices(tp, scale_mode):
    cfg = small_cfg()
    full = {n: M.synth_linear(SEED, "layers.0." + n, N, K, scale_mode)
            for n, N, K in (("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("v_proj", 1024, 4096),
                            ("o_proj", 4096, 4096), ("gate_proj", 12288, 4096), ("up_proj", 12288, 4096),
                            ("down_proj", 4096, 12288))}
    shards = [TP.layer_shard(TP.Partition(tp, r, cfg), SEED, 0, scale_mode, "cpu") for r in range(tp)]
    nq, nkv, ni = 4096 // tp, 1024 // tp, 12288 // tp
    b = lambda t: t.view(torch.uint8)
    # q|k|v rows: each rank's q rows, then its k rows, then its v rows
    for name, off, n, per in (("q_proj", 0, 4096, nq), ("k_proj", nq, 1024, nkv), ("v_proj", nq + nkv, 1024, nkv)):
        got = torch.cat([b(s["qkv"][0][off:off + per]) for s in shards])
        assert torch.equal(got, b(full[name][0])), name
    for name, off, per in (("gate_proj", 0, ni), ("up_proj", ni, ni)):
        got = torch.cat([b(s["gate_up"][0][off:off + per]) for s in shards])
        assert torch.equal(got, b(full[name][0])), name
    for name, key in (("o_proj", "o_proj"), ("down_proj", "down_proj")):
        got = torch.cat([b(s[key][0]) for s in shards], 1)
        assert torch.equal(got, b(full[name][0])), name
        if scale_mode == "block":
            assert torch.equal(torch.cat([s[key][1] for s in shards], 1), full[name][1])
        else:
            assert all(torch.equal(s[key][1], full[name][1]) for s in shards)


def test_partition_rejects_uneven_splits():
    with pytest.raises(ValueError):
        TP.Partition(3, 0, M.Config())
    with pytest.raises(ValueError):
        TP.Partition(2, 0, M.Config(vocab=1040))   # 520 rows per rank: not 16-aligned


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_w(sh, norms):
    return O.LayerW(norms["ln1"], norms["ln2"], norms["q"], norms["k"], *sh["qkv"], *sh["o_proj"], *sh["gate_up"],
                    *sh["down_proj"])


def _rank_main(rank, world, port, out_path):
    torch.set_num_threads(2)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = small_cfg()
        part = TP.Partition(world, rank, cfg)
        H, hd, ctx = 4096, 128, 40
        ones = torch.ones(H, dtype=torch.bfloat16)
        norms = {"ln1": ones, "ln2": ones, "q": torch.ones(hd, dtype=torch.bfloat16),
                 "k": torch.ones(hd, dtype=torch.bfloat16)}
        eps = 1e-6
        g = torch.Generator().manual_seed(3)
        h = torch.randn(H, generator=g).to(torch.bfloat16)
        kc_full = torch.randn(8, ctx + 1, hd, generator=g).to(torch.bfloat16)
        vc_full = torch.randn(8, ctx + 1, hd, generator=g).to(torch.bfloat16)
        cos, sin = M.rope_tables(ctx + 1, hd, 1e6, "cpu")
        sh = TP.layer_shard(part, SEED, 0, "channel", "cpu")
        ka, kb = part.kv_rows
        kc = kc_full[ka // hd:kb // hd].clone()
        vc = vc_full[ka // hd:kb // hd].clone()
        nq_l, nkv_l = 32 // world, 8 // world
        # one layer on the shard, with the TP engine's exchanges
        x = O.rms_norm(h[None], norms["ln1"], eps)
        qkv = O.fp8_linear(x, *sh["qkv"])[0]
        q, k, v = qkv.split([nq_l * hd, nkv_l * hd, nkv_l * hd])
        q = O.norm_rope(q.view(nq_l, hd), norms["q"], cos[ctx], sin[ctx], eps)
        k = O.norm_rope(k.view(nkv_l, hd), norms["k"], cos[ctx], sin[ctx], eps)
        kc[:, ctx] = k
        vc[:, ctx] = v.view(nkv_l, hd)
        attn = O.attention_f32(q, kc, vc, hd ** -0.5)
        part_o = O.fp8_linear_f32(attn[None].contiguous(), *sh["o_proj"])[0]
        dist.all_reduce(part_o)
        h1 = (h.float() + part_o.to(torch.bfloat16).float()).to(torch.bfloat16)
        x = O.rms_norm(h1[None], norms["ln2"], eps)
        gu = O.fp8_linear(x, *sh["gate_up"])[0]
        gt, up = gu.split([gu.shape[0] // 2] * 2)
        a = torch.nn.functional.silu(gt) * up
        part_d = O.fp8_linear_f32(a[None].contiguous(), *sh["down_proj"])[0]
        dist.all_reduce(part_d)
        h2 = (h1.float() + part_d.to(torch.bfloat16).float()).to(torch.bfloat16)
        # vocab-parallel head: (value, -index) max over ranks = the global greedy token
        hw, hs = TP.head_shard(part, SEED, "fp8", "cpu")
        logits = O.lm_head_logits(h2, ones, hw, hs, eps).float()
        i_loc = int(logits.argmax())
        key = torch.tensor([logits[i_loc].item(), -(part.vocab_rows[0] + i_loc)], dtype=torch.float64)
        keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(keys, key)
        best = max(keys, key=lambda t: (t[0].item(), t[1].item()))
        tok = int(-best[1].item())
        if rank == 0:
            # unsharded oracle on the same full weights
            full = TP.layer_shard(TP.Partition(1, 0, cfg), SEED, 0, "channel", "cpu")
            kcf, vcf = kc_full.clone(), vc_full.clone()
            ref = O.decode_layer(h, _layer_w(full, norms), kcf, vcf, ctx, cos, sin, eps)
            fw, fs = TP.head_shard(TP.Partition(1, 0, cfg), SEED, "fp8", "cpu")
            ref_tok = O.argmax_lowest(O.lm_head_logits(ref, ones, fw, fs, eps))
            rel = ((h2.float() - ref.float()).norm() / ref.float().norm()).item()
            torch.save({"rel": rel, "tok": tok, "ref_tok": ref_tok,
                        "k_rows": torch.equal(kc[:, ctx], kcf[ka // hd:kb // hd, ctx])}, out_path)
    finally:
        dist.destroy_process_group()


def test_tp2_layer_matches_unsharded_oracle(tmp_path):
    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn", join=True)
    r = torch.load(out)
    assert r["k_rows"], "the rank's K rows differ from the unsharded layer's"
    assert r["rel"] < 1e-2, r          # equal up to the order of the fp32 partial sums
    assert r["tok"] == r["ref_tok"], r
