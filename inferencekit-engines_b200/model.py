"""Qwen3-8B FP8 decode model state for the B200 kernels: config, weights, KV cache, RoPE tables.

Mirrors the decode-relevant half of the reference loader (qwen3-8b-fp8_rtx-5090/model.py):

* `Config` and `check_supported` follow model.py:27-89 (shapes compiled into the kernels).
* q|k|v and gate|up are row-concatenated like model.py:187-203.
* The KV cache is bf16 `[layer, kv_head, position, head_dim]` (model.py:208-211).
* RoPE tables are computed with the same torch ops as model.py:213-219 (fp32 angles, bf16 tables), on the
  device the engine runs on.

What differs is the FP8 weight layout. The reference re-tiles each matrix for register loads
(model.py:92-104). The B200 GEMV streams each warp's share of the weights through a shared-memory ring with
bulk async copies, then reads MMA fragments out of shared memory, so `pack_fp8` builds 2 KiB tiles (16 rows
x 128 k) that are conflict-free to read from shared memory (see `pack_fp8`).

Weights here are synthetic and seeded (no checkpoint in this environment): linear weights N(0, 0.02) in
fp32, quantized to float8_e4m3fn with either per-output-channel scales (absmax/448, the north-star format)
or 128x128 block scales (the reference checkpoint's format).
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field

import torch

from kernels import PackedFP8, PackedFP8Pairs, PackedTiles

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0
QBLOCK = 128

# Shapes compiled into the decode kernels (the same constants as the reference's KERNEL_SHAPES, model.py:27-31).
KERNEL_SHAPES = {"hidden_size": 4096, "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
                 "intermediate_size": 12288}


@dataclass
class Config:
    hidden: int = 4096
    layers: int = 36
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    inter: int = 12288
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1_000_000.0

    def check(self) -> None:
        """Raise ValueError unless the shapes are the ones the kernels are compiled for
        (the reference refuses other checkpoints the same way, model.py:34-67)."""
        got = {"hidden_size": self.hidden, "num_attention_heads": self.n_heads,
               "num_key_value_heads": self.n_kv_heads, "head_dim": self.head_dim,
               "intermediate_size": self.inter}
        bad = [f"{k} = {got[k]}, kernels are compiled for {v}" for k, v in KERNEL_SHAPES.items() if got[k] != v]
        if self.vocab % 16:
            bad.append(f"vocab_size = {self.vocab} must be a multiple of 16")
        if bad:
            raise ValueError("unsupported config:\n  - " + "\n  - ".join(bad))


# ------------------------------------------------------------------------------------------------------------
# Seeded synthetic weights
# ------------------------------------------------------------------------------------------------------------
def name_seed(seed: int, name: str) -> int:
    """Stable per-tensor seed: base seed plus a CRC of the tensor name."""
    return (seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF


def randn(shape, seed: int, name: str, device="cpu", std: float = 1.0) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(name_seed(seed, name))
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    return t.mul_(std) if std != 1.0 else t


def quantize_fp8(w: torch.Tensor, scale_mode: str):
    """fp32 [N, K] -> (fp8 [N, K], fp32 scales). scale_mode "channel": one scale per output row,
    absmax/448 (shape [N]); "block": one scale per 128x128 block (shape [N/128, K/128])."""
    N, K = w.shape
    if scale_mode == "channel":
        s = w.abs().amax(dim=1) / FP8_MAX
        s = torch.where(s > 0, s, torch.ones_like(s))
        q = (w / s[:, None]).clamp_(-FP8_MAX, FP8_MAX).to(FP8)
        return q, s.contiguous()
    if scale_mode == "block":
        assert N % QBLOCK == 0 and K % QBLOCK == 0
        b = w.view(N // QBLOCK, QBLOCK, K // QBLOCK, QBLOCK)
        s = b.abs().amax(dim=(1, 3)) / FP8_MAX
        s = torch.where(s > 0, s, torch.ones_like(s))
        q = (b / s[:, None, :, None]).clamp_(-FP8_MAX, FP8_MAX).to(FP8).view(N, K)
        return q, s.contiguous()
    raise ValueError(f"unknown scale_mode {scale_mode!r}")


def synth_linear(seed: int, name: str, N: int, K: int, scale_mode: str, device="cpu", std: float = 0.02):
    return quantize_fp8(randn((N, K), seed, name, device, std), scale_mode)


def synth_norm(seed: int, name: str, n: int, init: str, device="cpu") -> torch.Tensor:
    if init == "ones":
        return torch.ones(n, dtype=torch.bfloat16, device=device)
    return (1.0 + randn((n,), seed, name, device, 0.1)).to(torch.bfloat16)


# ------------------------------------------------------------------------------------------------------------
# FP8 weight layout for the GEMV kernels
# ------------------------------------------------------------------------------------------------------------
def pack_fp8(w: torch.Tensor, pairs: bool = False) -> torch.Tensor:
    """Row-major fp8 [N, K] -> the packed uint8 layout the B200 GEMV streams.

    A unit is 16 output rows (for `pairs`, 16 gate rows + the matching 16 up rows, gate|up stacked as
    [2I, K]). For unit u and 128-wide K block kb there is one 2 KiB tile per 16 rows:

        tile[c][lane][16 bytes],  c = 32-wide K chunk (0..3), lane = 4*g + t (g = 0..7, t = 0..3)
        the 16 bytes are words (hi, hh) in the order (0,0) (0,1) (1,0) (1,1), each holding
        row 16u + 8*hh + g, k = 128*kb + 32*c + 16*hi + 4*t + (0..3)

    i.e. lane L's 16 bytes are exactly its A-operand registers for the two m16n8k16 MMAs of chunk c with
    rows g and g+8 (see fp8_chunk_dot in csrc/common.cuh); that mapping is fixed by the MMA's fragment
    layout. [c][lane] order makes a warp's 16-byte shared-memory reads contiguous (no bank conflicts).
    Tiles are ordered [unit][kb] (for pairs [unit][kb][gate, up]), so the tiles of consecutive units are
    one contiguous stream and any split of that stream into ranges is a contiguous byte range.
    """
    N, K = w.shape
    assert w.dtype == FP8 and N % 16 == 0 and K % QBLOCK == 0
    w = w.as_subclass(torch.Tensor)
    KB = K // QBLOCK
    u8 = w.contiguous().view(torch.uint8)
    if pairs:
        assert N % 32 == 0
        half = N // 2
        g = pack_fp8(w[:half]).as_subclass(torch.Tensor).view(half // 16, KB, 1, 2048)
        u = pack_fp8(w[half:]).as_subclass(torch.Tensor).view(half // 16, KB, 1, 2048)
        return torch.cat([g, u], dim=2).reshape(-1).contiguous().as_subclass(PackedFP8Pairs)
    # element (n, k): n = 16*u + 8*hh + g, k = 128*kb + 32*c + 16*hi + 4*t + b
    v = u8.view(N // 16, 2, 8, KB, 4, 2, 4, 4)           # [u, hh, g, kb, c, hi, t, b]
    v = v.permute(0, 3, 4, 2, 6, 5, 1, 7)                 # [u, kb, c, g, t, hi, hh, b]
    return v.contiguous().view(-1).as_subclass(PackedFP8)


def _tile_swizzle_index(device):
    """[128, 8] chunk gather index of one tile: row r's chunk position c holds source chunk c ^ (r % 8)."""
    r = torch.arange(128, device=device)[:, None]
    c = torch.arange(8, device=device)[None, :]
    return r.expand(128, 8), (c ^ (r % 8))


def pack_fp8_tiles(w: torch.Tensor) -> torch.Tensor:
    """Row-major fp8 [N, K] -> the tcgen05 linear's tile-packed layout (`qk_fp8_gemm_tiles`), same bytes:
    [N/128][K/128] tiles of 128 rows x 128 k (16 KiB), tile-major; inside a tile row r at byte 128 r with its
    16-byte chunk c stored at chunk position c ^ (r % 8) (the 128-byte swizzle). Returned as an fp8 [N, K]
    `PackedTiles` tensor."""
    N, K = w.shape
    assert N % 128 == 0 and K % 128 == 0, (N, K)
    v = w.contiguous().view(torch.uint8).view(N // 128, 128, K // 128, 8, 16).permute(0, 2, 1, 3, 4)  # [t, kb, r, c, b]
    ri, ci = _tile_swizzle_index(w.device)
    out = v[:, :, ri, ci, :]               # out[.., r, c'] = in[.., r, c' ^ (r % 8)]
    return out.contiguous().view(FP8).view(N, K).as_subclass(PackedTiles)


def unpack_fp8_tiles(p: torch.Tensor) -> torch.Tensor:
    """Inverse of pack_fp8_tiles (tests)."""
    N, K = p.shape
    v = p.as_subclass(torch.Tensor).contiguous().view(torch.uint8).view(N // 128, K // 128, 128, 8, 16)
    ri, ci = _tile_swizzle_index(p.device)
    v = v[:, :, ri, ci, :]                 # the swizzle is its own inverse
    return v.permute(0, 2, 1, 3, 4).contiguous().view(FP8).view(N, K)


def pack_reference_tiled(wt: torch.Tensor, kmajor: bool, pairs: bool = False) -> torch.Tensor:
    """Weights in the reference's mma-tiled layout (qwen3-8b-fp8_rtx-5090/model.py:92-104, `tile_fp8`, fp8
    [N, K]) -> `pack_fp8` layout. That layout groups 8 rows and 64-wide K chunks into 512-byte tiles, either
    group-major ([ng, kc, g, t, q, b]) or K-major ([kc, ng, g, t, q, b]), with element (n, k) at
    n = 8*ng + g, k = 64*kc + 16*q + 4*t + b; undoing that order gives the row-major matrix."""
    N, K = wt.shape
    v = wt.as_subclass(torch.Tensor).contiguous().view(torch.uint8)
    if kmajor:
        v = v.view(K // 64, N // 8, 8, 4, 4, 4).permute(1, 2, 0, 4, 3, 5)   # -> [ng, g, kc, q, t, b]
    else:
        v = v.view(N // 8, K // 64, 8, 4, 4, 4).permute(0, 2, 1, 4, 3, 5)
    return pack_fp8(v.contiguous().view(N, K).view(FP8), pairs)


def unpack_fp8(p: torch.Tensor, N: int, K: int, pairs: bool = False) -> torch.Tensor:
    """Inverse of pack_fp8 (tests and TP re-sharding)."""
    KB = K // QBLOCK
    p = p.as_subclass(torch.Tensor)
    if pairs:
        half = N // 2
        v = p.view(torch.uint8).view(half // 16, KB, 2, 2048)
        g = unpack_fp8(v[:, :, 0].contiguous().view(-1), half, K)
        u = unpack_fp8(v[:, :, 1].contiguous().view(-1), half, K)
        return torch.cat([g, u], 0)
    v = p.view(torch.uint8).view(N // 16, KB, 4, 8, 4, 2, 2, 4)  # [u, kb, c, g, t, hi, hh, b]
    v = v.permute(0, 6, 3, 1, 2, 5, 4, 7)                       # [u, hh, g, kb, c, hi, t, b]
    return v.contiguous().view(N, K).view(FP8)


def quantize_kv_rows(x: torch.Tensor):
    """bf16 rows [..., 128] -> (e4m3 [..., 128], fp32 scales [...]): s = amax / 448, q = e4m3(x / s) round to
    nearest even, saturating, s = 0 -> 0 (the FP8 KV cache's row format; the kernels divide with div.full, so
    a quotient at a rounding tie can land one e4m3 step away). For cache set-up and tests."""
    xf = x.float()
    s = xf.abs().amax(-1) / FP8_MAX
    safe = torch.where(s > 0, s, torch.ones_like(s))
    q = torch.where(s[..., None] > 0, xf / safe[..., None], torch.zeros_like(xf))
    return q.clamp(-FP8_MAX, FP8_MAX).to(FP8), s


def rope_tables(max_seq: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin tables [max_seq, head_dim], same ops as the reference (model.py:213-219)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(max_seq, device=device).float()
    freqs = pos[:, None] * inv_freq.to(device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


# ------------------------------------------------------------------------------------------------------------
# Model container
# ------------------------------------------------------------------------------------------------------------
class Layer:
    """One decoder layer's decode-step weights (packed fp8 + fp32 scales + bf16 norms)."""


@dataclass
class Linear:
    packed: torch.Tensor        # PackedFP8 (uint8, pack_fp8 layout)
    scale: torch.Tensor         # fp32 [N] (channel) or [N/128, K/128] (block)
    N: int
    K: int
    pairs: bool = False

    @property
    def scale_mode(self) -> str:
        return "channel" if self.scale.dim() == 1 else "block"


@dataclass
class Qwen3FP8Decode:
    """Weights + KV cache + RoPE tables of the decode step (one GPU, or one TP rank's shard)."""
    cfg: Config
    max_seq: int
    device: str
    scale_mode: str = "channel"
    head_dtype: str = "fp8"       # "fp8" (per-channel scales) or "bf16" (reference format)
    kv_dtype: str = "bf16"        # "bf16" (the reference's cache) or "fp8" (e4m3 rows + fp32 row scales)
    layers: list = field(default_factory=list)
    batch: int = 1

    @staticmethod
    def synthetic(cfg: Config, max_seq: int = 4096, device: str = "cuda", seed: int = 0,
                  scale_mode: str = "channel", head_dtype: str = "fp8", norm_init: str = "ones",
                  n_layers: int | None = None, batch: int = 1, keep_rowmajor: bool = False) -> "Qwen3FP8Decode":
        """Random-init model with the Qwen3-8B shapes; every tensor is seeded by (seed, name).
        keep_rowmajor also keeps the row-major fp8 matrices (for oracle comparisons in tests)."""
        cfg.check()
        m = Qwen3FP8Decode(cfg, max_seq, device, scale_mode, head_dtype, batch=batch)
        H, I, hd = cfg.hidden, cfg.inter, cfg.head_dim
        nq, nkv = cfg.n_heads, cfg.n_kv_heads
        m.embed = randn((cfg.vocab, H), seed, "embed", device, 0.02).to(torch.bfloat16)
        m.norm = synth_norm(seed, "norm", H, norm_init, device)
        for li in range(cfg.layers if n_layers is None else n_layers):
            p = f"layers.{li}."
            L = Layer()
            L.ln1 = synth_norm(seed, p + "ln1", H, norm_init, device)
            L.ln2 = synth_norm(seed, p + "ln2", H, norm_init, device)
            L.q_norm = synth_norm(seed, p + "q_norm", hd, norm_init, device)
            L.k_norm = synth_norm(seed, p + "k_norm", hd, norm_init, device)
            L.rowmajor = {}

            def lin(name, N, K, pairs=False, parts=None):
                if parts is None:
                    q, s = synth_linear(seed, p + name, N, K, scale_mode, device)
                else:   # fused from separately seeded parts, like q|k|v and gate|up
                    qs = [synth_linear(seed, p + nm, n, K, scale_mode, device) for nm, n in parts]
                    q = torch.cat([a for a, _ in qs], 0)
                    s = torch.cat([b for _, b in qs], 0).contiguous()
                if keep_rowmajor:
                    L.rowmajor[name] = q
                return Linear(pack_fp8(q, pairs), s, N, K, pairs)

            L.qkv = lin("qkv", (nq + 2 * nkv) * hd, H,
                        parts=[("q_proj", nq * hd), ("k_proj", nkv * hd), ("v_proj", nkv * hd)])
            L.o = lin("o_proj", H, nq * hd)
            L.gu = lin("gate_up", 2 * I, H, pairs=True, parts=[("gate_proj", I), ("up_proj", I)])
            L.down = lin("down_proj", H, I)
            m.layers.append(L)
        if head_dtype == "fp8":
            q, s = quantize_fp8(randn((cfg.vocab, H), seed, "lm_head", device, 0.02), "channel")
            m.lm_head = Linear(pack_fp8(q), s, cfg.vocab, H)
            m.lm_head_rowmajor = q if keep_rowmajor else None
        else:
            m.lm_head = randn((cfg.vocab, H), seed, "lm_head", device, 0.02).to(torch.bfloat16)
            m.lm_head_rowmajor = m.lm_head
        m.alloc_cache()
        return m

    @staticmethod
    def from_weights(cfg: Config, layers: list, embed: torch.Tensor, norm: torch.Tensor, lm_head: torch.Tensor,
                     lm_head_scale: torch.Tensor | None = None, max_seq: int = 4096, device: str = "cuda",
                     batch: int = 1) -> "Qwen3FP8Decode":
        """Build from row-major weights. layers: dicts with ln1, ln2, q_norm, k_norm (bf16) and
        qkv, o_proj, gate_up, down_proj = (fp8 [N, K], fp32 scale) with q|k|v and gate|up concatenated.
        lm_head: bf16 [V, H], or fp8 [V, H] with lm_head_scale fp32 [V]."""
        scale_mode = "channel" if layers[0]["qkv"][1].dim() == 1 else "block"
        m = Qwen3FP8Decode(cfg, max_seq, device, scale_mode, "fp8" if lm_head_scale is not None else "bf16",
                           batch=batch)
        m.embed, m.norm = embed.to(device), norm.to(device)
        for d in layers:
            L = Layer()
            L.ln1, L.ln2, L.q_norm, L.k_norm = (d[k].to(device) for k in ("ln1", "ln2", "q_norm", "k_norm"))
            L.rowmajor = {}
            for attr, name, pairs in (("qkv", "qkv", False), ("o", "o_proj", False), ("gu", "gate_up", True),
                                      ("down", "down_proj", False)):
                w, s = d[name]
                setattr(L, attr, Linear(pack_fp8(w, pairs).to(device), s.to(device), w.shape[0], w.shape[1], pairs))
            m.layers.append(L)
        if lm_head_scale is not None:
            m.lm_head = Linear(pack_fp8(lm_head).to(device), lm_head_scale.to(device), lm_head.shape[0], lm_head.shape[1])
        else:
            m.lm_head = lm_head.to(device)
        m.lm_head_rowmajor = None
        m.alloc_cache()
        return m

    def alloc_cache(self):
        cfg = self.cfg
        shape = (len(self.layers), self.batch, cfg.n_kv_heads, self.max_seq, cfg.head_dim)
        if self.kv_dtype == "fp8":   # e4m3 rows [.., 128] + one fp32 scale per row
            self.k_cache = torch.zeros(shape, dtype=torch.uint8, device=self.device)
            self.v_cache = torch.zeros(shape, dtype=torch.uint8, device=self.device)
            self.k_scale = torch.zeros(shape[:-1], dtype=torch.float32, device=self.device)
            self.v_scale = torch.zeros(shape[:-1], dtype=torch.float32, device=self.device)
        else:
            self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
            self.v_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
            self.k_scale = self.v_scale = None
        self.cos, self.sin = rope_tables(self.max_seq, cfg.head_dim, cfg.rope_theta, self.device)

    def set_kv_dtype(self, kv_dtype: str):
        """Reallocate the KV cache as "bf16" or "fp8" (zeroed; the cache's contents are not converted)."""
        if kv_dtype not in ("bf16", "fp8"):
            raise ValueError(f"kv_dtype must be bf16 or fp8, got {kv_dtype!r}")
        self.kv_dtype = kv_dtype
        self.alloc_cache()

    def fill_cache_random(self, upto: int, seed: int = 1234):
        """KV positions [0, upto) = N(0, 1) bf16 (the synthetic long-context setups), generated in slices; an
        FP8 cache gets those rows quantized (`quantize_kv_rows`)."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for li in range(len(self.layers)):
            for ci, c in enumerate((self.k_cache, self.v_cache)):
                t = c[li, :, :, :upto]
                x = torch.randn(t.shape, generator=g, device=self.device, dtype=torch.float32)
                if self.kv_dtype == "fp8":
                    q, sc = quantize_kv_rows(x.to(torch.bfloat16))
                    t.copy_(q.view(torch.uint8))
                    (self.k_scale, self.v_scale)[ci][li, :, :, :upto].copy_(sc)
                else:
                    t.copy_(x)

    def weight_bytes(self) -> dict:
        """Algorithmic bytes one decode token reads (weights, scales, norms, embedding row)."""
        lin = sum(L.qkv.packed.numel() + L.o.packed.numel() + L.gu.packed.numel() + L.down.packed.numel()
                  for L in self.layers)
        scales = sum(4 * (L.qkv.scale.numel() + L.o.scale.numel() + L.gu.scale.numel() + L.down.scale.numel())
                     for L in self.layers)
        if isinstance(self.lm_head, Linear):
            head = self.lm_head.packed.numel() + 4 * self.lm_head.scale.numel()
        else:
            head = self.lm_head.numel() * 2
        norms = sum(2 * (2 * self.cfg.hidden + 2 * self.cfg.head_dim) for _ in self.layers) + 2 * self.cfg.hidden
        return {"linear": lin, "scales": scales, "head": head, "norms": norms, "embed_row": 2 * self.cfg.hidden}

    def kv_bytes_per_token(self, ctx: int) -> int:
        return len(self.layers) * self.cfg.n_kv_heads * self.cfg.head_dim * 2 * 2 * ctx


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def roofline_tok_s(bytes_per_token: float, gbs: float) -> float:
    return gbs * 1e9 / bytes_per_token if bytes_per_token else math.inf
