"""Generate the golden fixtures in this folder from the reference's own Python forward pass.

Runs ONLY where the reference checkout exists (it is read, never modified):
    python tests/golden/make_golden.py [--ref <reference checkout>/qwen3-8b-fp8_rtx-5090]
(default: oracle/refpath.py's engine_dir(), i.e. $QK_REFERENCE_DIR or a `reference` folder beside the repo)

What it does: imports the reference's `model.py` (qwen3-8b-fp8_rtx-5090/model.py), replaces its module-level
`fp8_linear` (imported from the Triton kernels at model.py:18) with the CPU restatement in
oracle/qwen3_ref.py, builds a `Qwen3FP8` object around seeded synthetic weights (bypassing the safetensors
loader, model.py:155-233) and calls the reference's `forward(tokens, start)` (model.py:243-281) on CPU for
single-token decode steps and one multi-token prefill. Everything except the FP8 GEMM arithmetic is the reference's code: RMSNorm,
q/k norm, RoPE, KV-cache writes, SDPA attention, residuals, SwiGLU, lm_head.

Fixtures (bf16 tensors stored as uint16 bit patterns):
  cfg1_channel.npz  benchmark configuration 1: one layer, per-output-channel scales, input hidden N(0,1), KV 0..1023
                    N(0,1), new token at position 1024. Layer output + K/V rows written at 1024.
  cfg1_block.npz    the same with 128x128 block scales (the reference checkpoint's format).
  steps_block.npz   a 2-layer model (block scales, bf16 lm_head of 1024 rows): 6 teacher-forced prompt
                    tokens then 10 greedy steps, all through forward(M=1); tokens + every step's logits.
  prefill_block.npz the same model, a 24-token prompt through one forward(tokens, 0) (the batched prefill,
                    causal SDPA): the last position's logits and both layers' K/V rows 0..23.
Inputs are regenerated from seeds by the package's synthetic-weight generator; each fixture stores a
checksum of its inputs so a drift in generation is detected instead of silently changing the baseline.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "inferencekit-engines_b200"))

from oracle import qwen3_ref as O  # noqa: E402
from oracle import refpath  # noqa: E402
import model as M  # noqa: E402  (the package's synthetic generator)

sys.path.pop(0)  # keep the package's `model` out of the way of the reference's


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def checksum(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()[:32]


def load_reference(ref_dir: str):
    """Import the reference's model.py with its Triton GEMM swapped for the CPU restatement."""
    # the package's `model` and `kernels` share their names with the reference's modules: set them aside
    ours = {k: sys.modules.pop(k) for k in list(sys.modules) if k in ("model", "kernels") or k.startswith("kernels.")}
    sys.path.insert(0, ref_dir)
    try:
        import model as ref_model  # the reference's file
    finally:
        sys.path.remove(ref_dir)
        for k in [k for k in sys.modules if k in ("model", "kernels") or k.startswith("kernels.")]:
            sys.modules.pop(k)
        sys.modules.update(ours)
    ref_model.fp8_linear = O.fp8_linear
    return ref_model


def layer_inputs(seed: int, scale_mode: str, norm_init: str = "random"):
    """Seeded row-major weights of one layer, generated like Qwen3FP8Decode.synthetic (CPU)."""
    H, I, hd, nq, nkv = 4096, 12288, 128, 32, 8
    p = "layers.0."
    w = {}
    for name, parts in (("qkv", [("q_proj", nq * hd), ("k_proj", nkv * hd), ("v_proj", nkv * hd)]),
                        ("gate_up", [("gate_proj", I), ("up_proj", I)])):
        qs = [M.synth_linear(seed, p + nm, n, H, scale_mode) for nm, n in parts]
        w[name] = (torch.cat([a for a, _ in qs], 0), torch.cat([b for _, b in qs], 0).contiguous())
    w["o_proj"] = M.synth_linear(seed, p + "o_proj", H, nq * hd, scale_mode)
    w["down_proj"] = M.synth_linear(seed, p + "down_proj", H, I, scale_mode)
    norms = {n: M.synth_norm(seed, p + n, H if n.startswith("ln") else hd, norm_init)
             for n in ("ln1", "ln2", "q_norm", "k_norm")}
    return w, norms


def make_ref_object(ref_model, layers_w, embed, lm_head, norm, max_seq, eps=1e-6):
    """A reference Qwen3FP8 without its safetensors loader: fields filled the way __init__ fills them."""
    m = object.__new__(ref_model.Qwen3FP8)
    m.cfg = ref_model.Config(vocab=embed.shape[0], layers=len(layers_w), eps=eps)
    m.kmajor = True
    m.rowmajor_copy = True
    m._prefill_impl = "ref"
    m.last_prefill_path = None
    m.max_seq = max_seq
    m.device = "cpu"
    m.embed, m.norm, m.lm_head = embed, norm, lm_head
    m.layers = []
    for w, norms in layers_w:
        L = ref_model.Layer()
        L.ln1, L.ln2, L.q_norm, L.k_norm = norms["ln1"], norms["ln2"], norms["q_norm"], norms["k_norm"]
        # tiled copies are never read when the row-major copy exists (model.py:239-241)
        L.w_qkv, L.s_qkv, L.r_qkv = None, w["qkv"][1], w["qkv"][0]
        L.w_o, L.s_o, L.r_o = None, w["o_proj"][1], w["o_proj"][0]
        L.w_gu, L.s_gu, L.r_gu = None, w["gate_up"][1], w["gate_up"][0]
        L.w_d, L.s_d, L.r_d = None, w["down_proj"][1], w["down_proj"][0]
        m.layers.append(L)
    shape = (len(layers_w), 8, max_seq, 128)
    m.k_cache = torch.zeros(shape, dtype=torch.bfloat16)
    m.v_cache = torch.zeros(shape, dtype=torch.bfloat16)
    m.cos, m.sin = M.rope_tables(max_seq, 128, 1_000_000.0, "cpu")
    m._untile_buf = None
    return m


def cfg1(ref_model, scale_mode: str, out_path: str, seed: int = 0, pos: int = 1024):
    w, norms = layer_inputs(seed, scale_mode)
    hidden = M.randn((4096,), seed, "cfg1.hidden").to(torch.bfloat16)
    max_seq = pos + 16
    m = make_ref_object(ref_model, [(w, norms)], hidden[None].clone(),
                        torch.zeros(8, 4096, dtype=torch.bfloat16), torch.ones(4096, dtype=torch.bfloat16),
                        max_seq)
    g = torch.Generator().manual_seed(M.name_seed(seed, "cfg1.kv"))
    m.k_cache[0, :, :pos] = torch.randn(8, pos, 128, generator=g).to(torch.bfloat16)
    m.v_cache[0, :, :pos] = torch.randn(8, pos, 128, generator=g).to(torch.bfloat16)
    k0, v0 = m.k_cache.clone(), m.v_cache.clone()
    seen = {}
    real_rms = ref_model.rms_norm

    def spy(x, wt, eps):                 # record the input of the final norm = the layer output
        if wt is m.norm:
            seen["h"] = x.clone()
        return real_rms(x, wt, eps)
    ref_model.rms_norm = spy
    try:
        m.forward(torch.tensor([0]), pos)
    finally:
        ref_model.rms_norm = real_rms
    out = seen["h"][0]
    # the forward must have touched exactly one KV slot per head
    dk = (m.k_cache != k0).any(-1)[0]
    dv = (m.v_cache != v0).any(-1)[0]
    assert not dk[:, :pos].any() and not dk[:, pos + 1:].any(), "K written outside its slot"
    assert not dv[:, :pos].any() and not dv[:, pos + 1:].any(), "V written outside its slot"
    np.savez_compressed(
        out_path, seed=seed, pos=pos, max_seq=max_seq, scale_mode=scale_mode,
        inputs_sha=checksum(w["qkv"][0], w["gate_up"][0], w["o_proj"][0], w["down_proj"][0], hidden,
                            k0[0, :, :pos], v0[0, :, :pos], *norms.values()),
        out_resid=u16(out), k_row=u16(m.k_cache[0, :, pos]), v_row=u16(m.v_cache[0, :, pos]))
    print(f"wrote {out_path}: |out| {out.float().norm():.3f}")


def steps(ref_model, out_path: str, seed: int = 7, vocab: int = 1024, n_layers: int = 2,
          prompt=(11, 503, 7, 999, 64, 300), gen: int = 10):
    lw = []
    for li in range(n_layers):
        w, norms = layer_inputs(seed + li, "block")
        lw.append((w, norms))
    embed = M.randn((vocab, 4096), seed, "steps.embed", std=1.0).to(torch.bfloat16)
    head = M.randn((vocab, 4096), seed, "steps.head", std=0.02).to(torch.bfloat16)
    norm = M.synth_norm(seed, "steps.norm", 4096, "random")
    max_seq = 32
    m = make_ref_object(ref_model, lw, embed, head, norm, max_seq)
    toks, logits = [], []
    cur = prompt[0]
    for i in range(len(prompt) + gen):
        lg = m.forward(torch.tensor([cur]), i)
        logits.append(u16(lg))
        nxt = int(lg.float().argmax())
        toks.append(nxt)
        cur = prompt[i + 1] if i + 1 < len(prompt) else nxt
    np.savez_compressed(out_path, seed=seed, vocab=vocab, n_layers=n_layers, prompt=np.array(prompt),
                        tokens=np.array(toks), logits=np.stack(logits),
                        inputs_sha=checksum(embed, head, norm, *[w["qkv"][0] for w, _ in lw]))
    print(f"wrote {out_path}: tokens {toks}")


def prefill(ref_model, out_path: str, seed: int = 7, vocab: int = 1024, n_layers: int = 2, P: int = 24):
    """The same 2-layer model as `steps`, a P-token prompt through ONE forward(tokens, 0) (the reference's
    batched prefill: causal SDPA, K/V rows 0..P-1 written per layer); the last position's logits and the K/V
    rows."""
    lw = []
    for li in range(n_layers):
        w, norms = layer_inputs(seed + li, "block")
        lw.append((w, norms))
    embed = M.randn((vocab, 4096), seed, "steps.embed", std=1.0).to(torch.bfloat16)
    head = M.randn((vocab, 4096), seed, "steps.head", std=0.02).to(torch.bfloat16)
    norm = M.synth_norm(seed, "steps.norm", 4096, "random")
    m = make_ref_object(ref_model, lw, embed, head, norm, 32)
    g = torch.Generator().manual_seed(M.name_seed(seed, "prefill.prompt"))
    prompt = torch.randint(0, vocab, (P,), generator=g)
    lg = m.forward(prompt, 0)
    assert m.last_prefill_path == "ref"
    np.savez_compressed(out_path, seed=seed, vocab=vocab, n_layers=n_layers, prompt=prompt.numpy(),
                        logits=u16(lg), k_rows=u16(m.k_cache[:, :, :P]), v_rows=u16(m.v_cache[:, :, :P]),
                        inputs_sha=checksum(embed, head, norm, *[w["qkv"][0] for w, _ in lw]))
    print(f"wrote {out_path}: argmax {int(lg.float().argmax())}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=refpath.engine_dir())
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    ref_model = load_reference(args.ref)
    cfg1(ref_model, "channel", os.path.join(HERE, "cfg1_channel.npz"))
    cfg1(ref_model, "block", os.path.join(HERE, "cfg1_block.npz"))
    steps(ref_model, os.path.join(HERE, "steps_block.npz"))
    prefill(ref_model, os.path.join(HERE, "prefill_block.npz"))


if __name__ == "__main__":
    main()
