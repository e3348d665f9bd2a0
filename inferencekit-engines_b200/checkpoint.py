"""Checkpoint loader: a Hugging Face `Qwen3-8B-FP8`-format directory into the B200 engine's model state.

Follows the reference loader (qwen3-8b-fp8_rtx-5090/model.py:34-67 `check_supported`, :81-89
`Config.from_json`, :155-233 `Qwen3FP8.__init__` / `_read_safetensors`):

* `config.json` is validated before any tensor is read: the shapes compiled into the kernels, plain RoPE
  with a `rope_theta` (either config layout, and both must agree when both are present), SiLU, no attention
  bias, no sliding window, an untied lm_head and the 128 x 128-block FP8 W8A8 dynamic-activation recipe.
  The vocabulary is the one relaxation: the reference's logits buffer fixes it at 151,936, while these
  kernels take any multiple of 16.
* Tensors come from `model.safetensors.index.json` (every shard it names) or a single `model.safetensors`,
  with the Hugging Face names: `model.embed_tokens.weight`, `model.norm.weight`, `lm_head.weight` (bf16),
  per layer `input_layernorm`, `post_attention_layernorm`, `self_attn.{q,k}_norm` (bf16) and the seven
  projections `self_attn.{q,k,v,o}_proj`, `mlp.{gate,up,down}_proj` as `.weight` (e4m3 [N, K]) plus
  `.weight_scale_inv` (bf16 or fp32 [ceil(N/128), ceil(K/128)], upcast to fp32, exactly).
* q|k|v and gate|up are row-concatenated (weights and scales), like model.py:187-203, then packed for the
  GEMV (`model.pack_fp8`). Every tensor of the checkpoint must be used; a missing or unused one is an error.

The result is the reference checkpoint's format on this engine: 128 x 128 block scales and a bf16 head,
the configuration the op path and the fused step reproduce bit for bit against the reference's decode
kernels.
"""
from __future__ import annotations

import json
import os

import torch

import model as M

FP8 = torch.float8_e4m3fn
# The kernels' compiled shapes (the reference's KERNEL_SHAPES, model.py:27-31, without its fixed vocabulary).
CHECKPOINT_SHAPES = dict(M.KERNEL_SHAPES)


def check_supported(c: dict, path: str = "") -> None:
    """Raise ValueError unless config.json `c` describes a model these kernels compute correctly."""
    bad = []
    for k, want in CHECKPOINT_SHAPES.items():
        if c.get(k) != want:
            bad.append(f"{k} = {c.get(k)!r}, the decode kernels are compiled for {want}")
    vocab = c.get("vocab_size")
    if not isinstance(vocab, int) or vocab <= 0 or vocab % 16:
        bad.append(f"vocab_size = {vocab!r}: must be a positive multiple of 16")
    rope = c.get("rope_scaling") or {}
    rp = c.get("rope_parameters") or {}
    for src, d in (("rope_scaling", rope), ("rope_parameters", rp)):
        rtype = d.get("rope_type", d.get("type", "default"))
        if rtype != "default":
            bad.append(f"{src}.rope_type = {rtype!r}: only plain RoPE (rope_theta, no scaling) is implemented")
    theta, theta_p = c.get("rope_theta"), rp.get("rope_theta")
    if not (theta or theta_p):
        bad.append("rope_theta missing")
    if theta and theta_p and float(theta) != float(theta_p):
        bad.append(f"rope_theta = {theta!r} but rope_parameters.rope_theta = {theta_p!r}")
    if c.get("hidden_act", "silu") != "silu":
        bad.append(f"hidden_act = {c.get('hidden_act')!r}, only silu is implemented")
    if c.get("attention_bias", False):
        bad.append("attention_bias = true is not implemented")
    if c.get("use_sliding_window", False):
        bad.append("use_sliding_window = true is not implemented")
    if c.get("tie_word_embeddings", False):
        bad.append("tie_word_embeddings = true is not supported (the lm_head must be its own bf16 tensor)")
    q = c.get("quantization_config") or {}
    if not (q.get("quant_method") == "fp8" and list(q.get("weight_block_size") or []) == [128, 128]
            and q.get("activation_scheme") == "dynamic"):
        bad.append(f"quantization_config = {q!r}: expected fp8, weight_block_size [128, 128], dynamic activations")
    if bad:
        raise ValueError(f"unsupported checkpoint {path}: this engine is built for Qwen3-8B FP8 "
                         "(block-128 W8A8) only.\n  - " + "\n  - ".join(bad))


def config_from_json(path: str) -> M.Config:
    """`M.Config` from `path/config.json`, after `check_supported`."""
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    check_supported(c, path)
    theta = c.get("rope_theta") or (c.get("rope_parameters") or {}).get("rope_theta")
    return M.Config(hidden=c["hidden_size"], layers=c["num_hidden_layers"], n_heads=c["num_attention_heads"],
                    n_kv_heads=c["num_key_value_heads"], head_dim=c["head_dim"], inter=c["intermediate_size"],
                    vocab=c["vocab_size"], eps=float(c["rms_norm_eps"]), rope_theta=float(theta))


class _Tensors:
    """The checkpoint's tensors by name, read on demand (one at a time, on the CPU) from their shards."""

    def __init__(self, path: str):
        from safetensors import safe_open
        self._open = safe_open
        index = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                self.where = dict(json.load(f)["weight_map"])
        elif os.path.exists(os.path.join(path, "model.safetensors")):
            with safe_open(os.path.join(path, "model.safetensors"), framework="pt", device="cpu") as f:
                self.where = {k: "model.safetensors" for k in f.keys()}
        else:
            raise FileNotFoundError(f"{path}: neither model.safetensors.index.json nor model.safetensors")
        self.path = path
        self.unused = set(self.where)
        self._files = {}

    def take(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"checkpoint {self.path} has no tensor {name!r}")
        if name not in self.unused:
            raise KeyError(f"tensor {name!r} read twice")
        self.unused.discard(name)
        fname = self.where[name]
        if fname not in self._files:
            self._files[fname] = self._open(os.path.join(self.path, fname), framework="pt", device="cpu")
        return self._files[fname].get_tensor(name)

    def close(self):
        self._files.clear()


def _expect(t: torch.Tensor, name: str, dtype, shape):
    if t.dtype != dtype or tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: {t.dtype} {tuple(t.shape)}, expected {dtype} {tuple(shape)}")


def load_checkpoint(path: str, max_seq: int = 4096, device: str = "cuda", batch: int = 1) -> M.Qwen3FP8Decode:
    """Read a Qwen3-8B-FP8-format checkpoint directory into a `Qwen3FP8Decode` (block scales, bf16 head)."""
    cfg = config_from_json(path)
    H, I, hd, V = cfg.hidden, cfg.inter, cfg.head_dim, cfg.vocab
    nq, nkv = cfg.n_heads, cfg.n_kv_heads
    T = _Tensors(path)
    bf = torch.bfloat16

    def vec(name, n):
        t = T.take(name)
        _expect(t, name, bf, (n,))
        return t

    def lin(p, parts):
        ws, ss = [], []
        for proj, N, K in parts:
            w, s = T.take(p + proj + ".weight"), T.take(p + proj + ".weight_scale_inv")
            _expect(w, p + proj + ".weight", FP8, (N, K))
            if s.dtype not in (torch.float32, bf) or tuple(s.shape) != ((N + 127) // 128, (K + 127) // 128):
                raise ValueError(f"{p}{proj}.weight_scale_inv: {s.dtype} {tuple(s.shape)}, expected fp32 or bf16 "
                                 f"{((N + 127) // 128, (K + 127) // 128)}")
            ws.append(w)
            ss.append(s.float())     # bf16 -> fp32 is exact
        w = torch.cat(ws, 0) if len(ws) > 1 else ws[0]
        s = torch.cat(ss, 0) if len(ss) > 1 else ss[0]
        return w.contiguous(), s.contiguous()

    try:
        embed = T.take("model.embed_tokens.weight")
        _expect(embed, "model.embed_tokens.weight", bf, (V, H))
        norm = vec("model.norm.weight", H)
        lm_head = T.take("lm_head.weight")
        _expect(lm_head, "lm_head.weight", bf, (V, H))
        layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            layers.append(dict(
                ln1=vec(p + "input_layernorm.weight", H), ln2=vec(p + "post_attention_layernorm.weight", H),
                q_norm=vec(p + "self_attn.q_norm.weight", hd), k_norm=vec(p + "self_attn.k_norm.weight", hd),
                qkv=lin(p, [("self_attn.q_proj", nq * hd, H), ("self_attn.k_proj", nkv * hd, H),
                            ("self_attn.v_proj", nkv * hd, H)]),
                o_proj=lin(p, [("self_attn.o_proj", H, nq * hd)]),
                gate_up=lin(p, [("mlp.gate_proj", I, H), ("mlp.up_proj", I, H)]),
                down_proj=lin(p, [("mlp.down_proj", H, I)])))
        if T.unused:
            raise ValueError(f"checkpoint {path}: unused tensors {sorted(T.unused)[:5]}")
    finally:
        T.close()
    return M.Qwen3FP8Decode.from_weights(cfg, layers, embed, norm, lm_head.contiguous(), None, max_seq=max_seq,
                                         device=device, batch=batch)
