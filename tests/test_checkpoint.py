"""Checkpoint loader (checkpoint.py) on synthetic Qwen3-8B-FP8-format directories.

The real checkpoint is not available here, so each test writes one with the reference's tensor names, dtypes
and shapes (full per-layer shapes, 1-2 layers, a small vocabulary): config.json, sharded safetensors and the
index. Checked: every packed weight, scale, norm and table equals what `from_weights` builds from the same
tensors (q|k|v and gate|up concatenated, bf16 block scales upcast exactly); each unsupported config field,
a missing tensor, an unused tensor and a wrong dtype or shape is refused with a clear error; and on the GPU a
loaded model decodes identically through the op path and the fused step.
"""
import json
import os

import pytest
import torch

import checkpoint as C
import model as M

FP8 = torch.float8_e4m3fn
H, I, NQ, NKV, HD = 4096, 12288, 32, 8, 128


def hf_config(layers=1, vocab=256, **over):
    c = {"architectures": ["Qwen3ForCausalLM"], "hidden_size": H, "num_hidden_layers": layers,
         "num_attention_heads": NQ, "num_key_value_heads": NKV, "head_dim": HD, "intermediate_size": I,
         "vocab_size": vocab, "rms_norm_eps": 1e-6, "rope_theta": 1000000, "hidden_act": "silu",
         "attention_bias": False, "use_sliding_window": False, "tie_word_embeddings": False,
         "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128],
                                 "activation_scheme": "dynamic", "fmt": "e4m3"}}
    c.update(over)
    return c


def rand_fp8(g, N, K):
    """Random finite e4m3 bytes (no NaN encodings), scaled like trained weights' codes."""
    mag = torch.randint(0, 0x70, (N, K), generator=g, dtype=torch.uint8)
    sign = torch.randint(0, 2, (N, K), generator=g, dtype=torch.uint8) << 7
    return (mag | sign).view(FP8)


def synth_tensors(layers, vocab, seed=0, scale_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16

    def vec(n):
        return (1 + 0.1 * torch.randn(n, generator=g)).to(bf)

    t = {"model.embed_tokens.weight": (0.02 * torch.randn(vocab, H, generator=g)).to(bf),
         "model.norm.weight": vec(H),
         "lm_head.weight": (0.02 * torch.randn(vocab, H, generator=g)).to(bf)}
    projs = {"self_attn.q_proj": (NQ * HD, H), "self_attn.k_proj": (NKV * HD, H), "self_attn.v_proj": (NKV * HD, H),
             "self_attn.o_proj": (H, NQ * HD), "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H),
             "mlp.down_proj": (H, I)}
    for i in range(layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = vec(H)
        t[p + "post_attention_layernorm.weight"] = vec(H)
        t[p + "self_attn.q_norm.weight"] = vec(HD)
        t[p + "self_attn.k_norm.weight"] = vec(HD)
        for name, (N, K) in projs.items():
            t[p + name + ".weight"] = rand_fp8(g, N, K)
            t[p + name + ".weight_scale_inv"] = (torch.rand(N // 128, K // 128, generator=g) * 1e-3 + 1e-4).to(scale_dtype)
    return t


def write_checkpoint(path, tensors, config, shards=2):
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    names = sorted(tensors)
    where = {}
    for s in range(shards):
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        part = {n: tensors[n].contiguous() for j, n in enumerate(names) if j % shards == s}
        save_file(part, os.path.join(path, fname))
        where.update({n: fname for n in part})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": where}, f)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f)
    return where


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("ckpt"))
    tensors = synth_tensors(1, 256)
    write_checkpoint(path, tensors, hf_config(1, 256))
    return path, tensors


def test_load_matches_from_weights(ckpt):
    path, t = ckpt
    m = C.load_checkpoint(path, max_seq=64, device="cpu")
    assert (m.cfg.layers, m.cfg.vocab, m.cfg.rope_theta, m.cfg.eps) == (1, 256, 1e6, 1e-6)
    assert m.scale_mode == "block" and m.head_dtype == "bf16"
    p = "model.layers.0."
    L = m.layers[0]
    cat = lambda *ns: torch.cat([t[p + n + ".weight"] for n in ns], 0)                  # noqa: E731
    scat = lambda *ns: torch.cat([t[p + n + ".weight_scale_inv"].float() for n in ns], 0)  # noqa: E731
    for lin, names, pairs in ((L.qkv, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), False),
                              (L.o, ("self_attn.o_proj",), False), (L.gu, ("mlp.gate_proj", "mlp.up_proj"), True),
                              (L.down, ("mlp.down_proj",), False)):
        w = cat(*names)
        assert torch.equal(lin.packed.view(torch.uint8), M.pack_fp8(w, pairs).view(torch.uint8))
        assert torch.equal(M.unpack_fp8(lin.packed, lin.N, lin.K, pairs).view(torch.uint8), w.view(torch.uint8))
        assert lin.scale.dtype == torch.float32 and torch.equal(lin.scale, scat(*names))
    assert torch.equal(L.ln1, t[p + "input_layernorm.weight"]) and torch.equal(L.k_norm, t[p + "self_attn.k_norm.weight"])
    assert torch.equal(m.embed, t["model.embed_tokens.weight"]) and torch.equal(m.lm_head, t["lm_head.weight"])
    assert tuple(m.k_cache.shape) == (1, 1, NKV, 64, HD)
    cos, sin = M.rope_tables(64, HD, 1e6, "cpu")
    assert torch.equal(m.cos, cos) and torch.equal(m.sin, sin)


def test_rope_parameters_layout_and_fp32_scales(tmp_path):
    """The newer config layout (rope_parameters.rope_theta) and fp32 scale tensors load the same way."""
    t = synth_tensors(1, 128, seed=1, scale_dtype=torch.float32)
    c = hf_config(1, 128)
    del c["rope_theta"]
    c["rope_parameters"] = {"rope_type": "default", "rope_theta": 500000.0}
    write_checkpoint(str(tmp_path), t, c, shards=1)
    m = C.load_checkpoint(str(tmp_path), max_seq=16, device="cpu")
    assert m.cfg.rope_theta == 500000.0
    assert torch.equal(m.layers[0].o.scale, t["model.layers.0.self_attn.o_proj.weight_scale_inv"])


@pytest.mark.parametrize("over,match", [
    ({"hidden_size": 5120}, "hidden_size"),
    ({"num_key_value_heads": 4}, "num_key_value_heads"),
    ({"intermediate_size": 11008}, "intermediate_size"),
    ({"vocab_size": 151937}, "vocab_size"),
    ({"rope_scaling": {"rope_type": "yarn", "factor": 4.0}}, "rope_type"),
    ({"rope_theta": None}, "rope_theta missing"),
    ({"rope_parameters": {"rope_theta": 10000.0}}, "rope_parameters.rope_theta"),
    ({"hidden_act": "gelu"}, "hidden_act"),
    ({"attention_bias": True}, "attention_bias"),
    ({"use_sliding_window": True}, "use_sliding_window"),
    ({"tie_word_embeddings": True}, "tie_word_embeddings"),
    ({"quantization_config": {"quant_method": "fp8", "weight_block_size": [1, 128], "activation_scheme": "dynamic"}},
     "quantization_config"),
    ({"quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128], "activation_scheme": "static"}},
     "quantization_config"),
])
def test_check_supported_refuses(over, match):
    with pytest.raises(ValueError, match=match):
        C.check_supported(hf_config(**over), "synthetic")


def test_check_supported_accepts_the_reference_config():
    C.check_supported(hf_config(36, 151936))


def test_missing_unused_and_malformed_tensors(ckpt, tmp_path):
    path, t = ckpt
    with open(os.path.join(path, "model.safetensors.index.json")) as f:
        where = json.load(f)["weight_map"]
    shards = sorted(set(where.values()))
    for s in shards:   # the same shard files, indexed three ways
        os.symlink(os.path.join(path, s), os.path.join(tmp_path, s))
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump(hf_config(1, 256), f)

    def index(wm):
        with open(os.path.join(tmp_path, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wm}, f)

    missing = dict(where)
    del missing["model.layers.0.self_attn.k_norm.weight"]
    index(missing)
    with pytest.raises(KeyError, match="k_norm"):
        C.load_checkpoint(str(tmp_path), max_seq=16, device="cpu")

    from safetensors.torch import save_file
    save_file({"model.layers.0.self_attn.rotary_emb.inv_freq": torch.ones(64)}, os.path.join(tmp_path, "extra.safetensors"))
    index({**where, "model.layers.0.self_attn.rotary_emb.inv_freq": "extra.safetensors"})
    with pytest.raises(ValueError, match="unused tensors"):
        C.load_checkpoint(str(tmp_path), max_seq=16, device="cpu")

    # a bf16 projection weight (an unquantized checkpoint) is refused by dtype
    bad = {"model.layers.0.mlp.down_proj.weight": torch.zeros(H, I, dtype=torch.bfloat16)}
    save_file(bad, os.path.join(tmp_path, "bad.safetensors"))
    index({**where, "model.layers.0.mlp.down_proj.weight": "bad.safetensors"})
    with pytest.raises(ValueError, match="down_proj.weight"):
        C.load_checkpoint(str(tmp_path), max_seq=16, device="cpu")


@pytest.mark.gpu
def test_loaded_checkpoint_decodes_identically_on_both_engines(tmp_path):
    from generate import Engine
    t = synth_tensors(2, 4096, seed=2)
    write_checkpoint(str(tmp_path), t, hf_config(2, 4096), shards=3)
    m = C.load_checkpoint(str(tmp_path), max_seq=256, device="cuda")
    prompt = list(range(5, 40, 3))
    ops_tokens = Engine(m).generate(prompt, 12)
    kc = m.k_cache.clone()
    m.k_cache.zero_()
    m.v_cache.zero_()
    fused_tokens = Engine(m, fused=True).generate(prompt, 12)
    assert ops_tokens == fused_tokens
    assert torch.equal(kc, m.k_cache)
