"""The fused decode step (one persistent kernel per token, csrc/step.cuh) against the op-by-op path: same tokens,
same logits, same KV cache and residual stream, bit for bit, eager and graph-replayed."""
import pytest
import torch

import model as M

pytestmark = pytest.mark.gpu


def build(n_layers, scale_mode, vocab=4096, max_seq=512, seed=3, head="fp8"):
    cfg = M.Config(layers=n_layers, vocab=vocab)
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=max_seq, device="cuda", seed=seed, scale_mode=scale_mode,
                                   head_dtype=head, norm_init="random")
    return m


def run_steps(m, fused, start_pos, steps, use_graph, token=7, fill=None):
    from generate import Engine
    m.k_cache.zero_()
    m.v_cache.zero_()
    if fill:
        m.fill_cache_random(fill, seed=11)
    eng = Engine(m, fused=fused)
    eng.token.fill_(token)
    eng.state.copy_(torch.tensor([start_pos, 0], dtype=torch.int32))
    if use_graph:
        eng.capture()
    logits = []
    for _ in range(steps):
        eng.step(1, use_graph)
        logits.append(eng.logits.clone())
    torch.cuda.synchronize()
    assert eng.k.device_error() == 0
    return (eng.out_tokens[:steps].tolist(), torch.stack(logits), m.k_cache.clone(), m.v_cache.clone(),
            eng.resid.clone(), eng.state.clone())


def assert_same(a, b):
    toks_a, lg_a, k_a, v_a, r_a, st_a = a
    toks_b, lg_b, k_b, v_b, r_b, st_b = b
    assert toks_a == toks_b
    assert torch.equal(st_a, st_b)
    assert torch.equal(lg_a.view(torch.int16), lg_b.view(torch.int16))
    assert torch.equal(k_a, k_b) and torch.equal(v_a, v_b)
    assert torch.equal(r_a.view(torch.int16), r_b.view(torch.int16))


@pytest.mark.parametrize("scale_mode", ["channel", "block"])
def test_fused_step_matches_op_by_op_small(scale_mode):
    m = build(2, scale_mode)
    ref = run_steps(m, fused=False, start_pos=0, steps=6, use_graph=False)
    got = run_steps(m, fused=True, start_pos=0, steps=6, use_graph=False)
    assert_same(got, ref)


def test_fused_step_bf16_head_matches_op_by_op():
    """The reference checkpoint's format: block-128 scales and the bf16 lm_head (vocabulary not a multiple of
    the 4-row ring stage per CTA), bit for bit against the op path."""
    m = build(2, "block", vocab=4112, head="bf16")
    ref = run_steps(m, fused=False, start_pos=40, steps=5, use_graph=True, fill=40)
    got = run_steps(m, fused=True, start_pos=40, steps=5, use_graph=True, fill=40)
    assert_same(got, ref)


def test_fused_step_long_context_and_graph():
    """Contexts that span many 64-key splits (prefilled cache), graph replay of the fused kernel."""
    m = build(2, "channel", max_seq=4096)
    ref = run_steps(m, fused=False, start_pos=3000, steps=4, use_graph=True, fill=3000)
    got = run_steps(m, fused=True, start_pos=3000, steps=4, use_graph=True, fill=3000)
    assert_same(got, ref)


def test_fused_step_across_a_split_boundary():
    """Positions 61..66: the new key moves from the last slot of split 0 into a new split 1 (the split count
    goes from 1 to 2 between two steps), eager launches."""
    m = build(2, "channel")
    ref = run_steps(m, fused=False, start_pos=61, steps=6, use_graph=False, fill=61)
    got = run_steps(m, fused=True, start_pos=61, steps=6, use_graph=False, fill=61)
    assert_same(got, ref)


def test_fused_step_at_the_end_of_a_16k_cache():
    """256 splits per KV head, and the last three positions of the cache (16381..16383), graph replay."""
    m = build(2, "channel", max_seq=16384)
    ref = run_steps(m, fused=False, start_pos=16381, steps=3, use_graph=True, fill=16381)
    got = run_steps(m, fused=True, start_pos=16381, steps=3, use_graph=True, fill=16381)
    assert_same(got, ref)


def test_fused_step_at_the_end_of_a_64k_cache():
    """The longest context the fused step takes: 1,024 splits per KV head, positions 65533..65535."""
    m = build(2, "channel", max_seq=65536)
    ref = run_steps(m, fused=False, start_pos=65533, steps=3, use_graph=True, fill=65533)
    got = run_steps(m, fused=True, start_pos=65533, steps=3, use_graph=True, fill=65533)
    assert_same(got, ref)


def test_fused_step_full_model():
    """All 36 layers and the 151,936-row FP8 head: 8 greedy steps at ~4k context, bit-identical."""
    cfg = M.Config()
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=4096, device="cuda", seed=0, scale_mode="channel", head_dtype="fp8")
    ref = run_steps(m, fused=False, start_pos=3900, steps=8, use_graph=True, fill=3900)
    got = run_steps(m, fused=True, start_pos=3900, steps=8, use_graph=True, fill=3900)
    assert_same(got, ref)
