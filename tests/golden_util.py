"""Helpers shared by the tests: rebuild the golden-fixture inputs from their seeds, bf16 <-> uint16."""
import hashlib
import os

import numpy as np
import torch

import model as M

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def checksum(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()[:32]


def layer_inputs(seed: int, scale_mode: str, norm_init: str = "random"):
    """Same generation as tests/golden/make_golden.py:layer_inputs (kept in step by the checksum)."""
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


def cfg1_inputs(fx):
    """Rebuild the inputs of a cfg1_*.npz fixture and verify their checksum."""
    seed, pos, max_seq = int(fx["seed"]), int(fx["pos"]), int(fx["max_seq"])
    w, norms = layer_inputs(seed, str(fx["scale_mode"]))
    hidden = M.randn((4096,), seed, "cfg1.hidden").to(torch.bfloat16)
    g = torch.Generator().manual_seed(M.name_seed(seed, "cfg1.kv"))
    kc = torch.zeros(8, max_seq, 128, dtype=torch.bfloat16)
    vc = torch.zeros(8, max_seq, 128, dtype=torch.bfloat16)
    kc[:, :pos] = torch.randn(8, pos, 128, generator=g).to(torch.bfloat16)
    vc[:, :pos] = torch.randn(8, pos, 128, generator=g).to(torch.bfloat16)
    sha = checksum(w["qkv"][0], w["gate_up"][0], w["o_proj"][0], w["down_proj"][0], hidden,
                   kc[:, :pos], vc[:, :pos], *norms.values())
    assert sha == str(fx["inputs_sha"]), "synthetic input generation drifted from the golden fixture"
    return dict(w=w, norms=norms, hidden=hidden, kc=kc, vc=vc, pos=pos, max_seq=max_seq)


def oracle_layer(O, inp):
    w, n = inp["w"], inp["norms"]
    return O.LayerW(n["ln1"], n["ln2"], n["q_norm"], n["k_norm"], w["qkv"][0], w["qkv"][1],
                    w["o_proj"][0], w["o_proj"][1], w["gate_up"][0], w["gate_up"][1],
                    w["down_proj"][0], w["down_proj"][1])
