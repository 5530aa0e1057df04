#!/usr/bin/env python3
"""Pack DeepSeek-V2-Lite-shaped weights into the tensors the B200 decode graph attaches.

Drop-in for the reference's fleet/pack_weights.py (the same entry points: ``Dims``, ``REAL_DIMS``,
``pack_all(model_dir, device, dims, layers, head)`` and the ``pack_*`` functions, with the same
packed key names), with the B200 layout and its own reader (``SafetensorsDir``: memory-mapped
shards, tensors copied straight to the device):

* every tensor is BF16, row-major ``[out, in]`` as nn.Linear stores it, so a batch-1 GEMV
  streams whole rows (the weight stream is a run of contiguous bulk copies, no tensor map);
* ``W_qkva`` fuses q_proj and kv_a_proj_with_mqa (reference pack_qkva, pack_weights.py:144-147);
* ``W_ukT`` [NH, D_C, D_N] is the absorbed key up-projection stored transposed, so the per-head
  product ``ql_nope[h] = q_nope[h] @ W_uk[h]`` is a GEMV over contiguous 256-byte rows (the
  reference keeps W_uk [NH, D_N, D_C], pack_weights.py:150-161); ``W_uv`` [NH, D_V, D_C] as is;
* the MoE experts are ``W13`` [E_TOTAL, 2*I_MOE, H] and ``W2`` [E_TOTAL, H, I_MOE], with the shared
  MLP split into experts E and E+1 (the reference's D6, pack_weights.py:187-210); W13's gate and
  up rows are interleaved (row 2i gate i, row 2i+1 up i; the reference stacks gate rows then up
  rows) so a weight stage holds whole pairs and the SwiGLU is computed in the same task;
* layer 0's dense MLP is ``W_gu`` [2*I_DENSE, H] (interleaved the same way) and ``W_down``
  [H, I_DENSE]: no padding to 11,264 and no row shuffle, which only the reference's CK tile
  kernels needed (pack_weights.py:164-184).

``synthetic_packed`` makes the seeded random weights the benchmark configs use (BF16 ~N(0, 0.02),
norm weights 1.0), generated on the target device in a fixed tensor order.
"""
import argparse
import json
import math
from dataclasses import dataclass
from pathlib import Path

import torch

CHECKPOINT_BYTES = 31_412_968_448


@dataclass(frozen=True)
class Dims:
    H: int          # hidden_size
    NH: int         # num_attention_heads
    D_N: int        # qk_nope_head_dim
    D_R: int        # qk_rope_head_dim
    D_V: int        # v_head_dim
    D_C: int        # kv_lora_rank
    V: int          # vocab_size
    L: int          # num_hidden_layers
    I_DENSE: int    # intermediate_size (layer 0)
    I_MOE: int      # moe_intermediate_size
    E: int          # n_routed_experts
    TOPK: int       # num_experts_per_tok
    N_SHARED: int   # n_shared_experts

    @classmethod
    def from_config(cls, cfg):
        get = (lambda k: getattr(cfg, k)) if not isinstance(cfg, dict) else (lambda k: cfg[k])
        return cls(
            H=get("hidden_size"), NH=get("num_attention_heads"),
            D_N=get("qk_nope_head_dim"), D_R=get("qk_rope_head_dim"),
            D_V=get("v_head_dim"), D_C=get("kv_lora_rank"), V=get("vocab_size"),
            L=get("num_hidden_layers"), I_DENSE=get("intermediate_size"),
            I_MOE=get("moe_intermediate_size"), E=get("n_routed_experts"),
            TOPK=get("num_experts_per_tok"), N_SHARED=get("n_shared_experts"),
        )

    def to_dict(self):
        return {k: getattr(self, k) for k in self.__dataclass_fields__}

    @property
    def Q_OUT(self):
        return self.NH * (self.D_N + self.D_R)

    @property
    def KVA_OUT(self):
        return self.D_C + self.D_R

    @property
    def QKVA_OUT(self):
        return self.Q_OUT + self.KVA_OUT

    @property
    def KVB_OUT(self):
        return self.NH * (self.D_N + self.D_V)

    @property
    def E_TOTAL(self):
        return self.E + self.N_SHARED

    @property
    def I_SHARED(self):
        return self.I_MOE * self.N_SHARED

    @property
    def N_SLOTS(self):
        return self.TOPK + self.N_SHARED


REAL_DIMS = Dims(H=2048, NH=16, D_N=128, D_R=64, D_V=128, D_C=512, V=102400, L=27,
                 I_DENSE=10944, I_MOE=1408, E=64, TOPK=6, N_SHARED=2)


def check_tiling(d: Dims):
    """What the sm_100a task kernels require of the shapes (all of them hold at REAL_DIMS):
    every GEMV row is a whole number of 16-byte vectors, the RoPE width is even, and the
    per-lane activation slice of a GEMV (K / 256 vectors of 8) fits the 8-vector register file."""
    for k in (d.H, d.D_N, d.D_C, d.I_MOE, d.I_DENSE, d.NH * d.D_V):
        assert k % 8 == 0, f"GEMV K {k} must be a multiple of 8 BF16 (16-byte rows)"
    assert d.D_R % 2 == 0 and d.D_R <= 128
    assert d.H <= 2048 and d.I_MOE <= 2048 and d.D_C <= 2048, "K beyond 2048 needs the K-split form"
    assert d.D_C % 32 == 0 and d.D_R % 8 == 0
    assert d.N_SLOTS <= 8 and d.E_TOTAL <= 256


# ----------------------------------------------------------------------------
# packing: one builder per packed tensor, over a getter of the layer's checkpoint tensors
#
# Every builder takes get(suffix) -> the layer's tensor named model.layers.{l}.<suffix> (BF16,
# [out, in] as nn.Linear stores it), so a state dict and a checkpoint on disk pack through the
# same code. The packed key names and shapes are the loader's interface (the graph attaches them).


def _rows_of(parts):
    """The row-wise concatenation of 2-D tensors into one new contiguous tensor."""
    out = torch.empty(sum(int(t.shape[0]) for t in parts), int(parts[0].shape[1]), dtype=parts[0].dtype,
                      device=parts[0].device)
    r = 0
    for t in parts:
        out[r:r + t.shape[0]].copy_(t)
        r += t.shape[0]
    return out


def pack_qkva(w_q, w_kva):
    """[Q_OUT + KVA_OUT, H]: q_proj's rows (head-major, nope then rope), then kv_a_proj_with_mqa's
    (the 512 latent rows, then the 64 rope rows)."""
    if w_q.shape[1] != w_kva.shape[1]:
        raise ValueError(f"q_proj {tuple(w_q.shape)} and kv_a_proj {tuple(w_kva.shape)} disagree on H")
    return _rows_of([w_q, w_kva])


def split_uk_uv(d: Dims, w_kvb, contiguous=False):
    """kv_b_proj [NH * (D_N + D_V), D_C] as its two per-head blocks W_uk [NH, D_N, D_C] and
    W_uv [NH, D_V, D_C] (views unless contiguous): k_nope[h] = W_uk[h] c, v[h] = W_uv[h] c."""
    if tuple(w_kvb.shape) != (d.KVB_OUT, d.D_C):
        raise ValueError(f"kv_b_proj {tuple(w_kvb.shape)}, expected {(d.KVB_OUT, d.D_C)}")
    w_uk, w_uv = w_kvb.unflatten(0, (d.NH, d.D_N + d.D_V)).split([d.D_N, d.D_V], dim=1)
    return (w_uk.contiguous(), w_uv.contiguous()) if contiguous else (w_uk, w_uv)


def transpose_uk(w_uk):
    """W_uk [NH, D_N, D_C] -> W_ukT [NH, D_C, D_N]: one contiguous row per latent column."""
    return w_uk.transpose(1, 2).contiguous()


def interleave_gate_up(gate, up):
    """[I, K] gate and up -> [2I, K] with row 2i = gate row i and row 2i + 1 = up row i, so one
    weight stage holds whole (gate, up) pairs and the SwiGLU fuses into the GEMV."""
    assert gate.shape == up.shape
    return torch.stack([gate, up], dim=1).reshape(2 * gate.shape[0], *gate.shape[1:]).contiguous()


def deinterleave_gate_up(w):
    """Inverse of interleave_gate_up: [2I, K] -> (gate [I, K], up [I, K])."""
    return w[0::2], w[1::2]


def pack_dense_mlp(d: Dims, w_gate, w_up, w_down):
    """Layer 0: W_gu [2*I_DENSE, H] with gate and up rows interleaved; W_down [H, I_DENSE]."""
    assert w_gate.shape == (d.I_DENSE, d.H) and w_up.shape == (d.I_DENSE, d.H)
    assert w_down.shape == (d.H, d.I_DENSE)
    return {"W_gu": interleave_gate_up(w_gate, w_up), "W_down": w_down.contiguous()}


def pack_moe(d: Dims, w_gate_router, experts, shared):
    """W13 [E_TOTAL, 2*I_MOE, H] (gate and up rows interleaved) and W2 [E_TOTAL, H, I_MOE]: the E
    routed experts, then the shared MLP cut into N_SHARED experts of I_MOE intermediate rows each
    (expert E + s takes the shared gate/up rows [s*I_MOE, (s+1)*I_MOE) and the same down columns:
    the always-selected experts of the graph). experts: E triples (gate, up, down)."""
    if tuple(w_gate_router.shape) != (d.E, d.H) or len(experts) != d.E:
        raise ValueError(f"router {tuple(w_gate_router.shape)} / {len(experts)} experts for E = {d.E}")
    sg, su, sd = shared
    if tuple(sg.shape) != (d.I_SHARED, d.H) or tuple(su.shape) != (d.I_SHARED, d.H) or tuple(sd.shape) != (d.H, d.I_SHARED):
        raise ValueError("shared expert shapes")
    triples = list(experts) + [(sg[k * d.I_MOE:(k + 1) * d.I_MOE], su[k * d.I_MOE:(k + 1) * d.I_MOE],
                                sd[:, k * d.I_MOE:(k + 1) * d.I_MOE]) for k in range(d.N_SHARED)]
    for g, u, dn in triples:
        if tuple(g.shape) != (d.I_MOE, d.H) or tuple(u.shape) != (d.I_MOE, d.H) or tuple(dn.shape) != (d.H, d.I_MOE):
            raise ValueError("expert shapes")
    return {"W_gate": w_gate_router.contiguous(),
            "W13": torch.stack([interleave_gate_up(g, u) for g, u, _ in triples]),
            "W2": torch.stack([dn.contiguous() for _, _, dn in triples])}


# ----------------------------------------------------------------------------
# the down projection regrouped by expert unit (include/fleet_mk.h MK_OP_MOE_UNITS)


def unit_parts(i):
    """Parts of a down-projection row of i values (the row engine's: the fewest of 1, 2, 4, 8 with
    at most 256 values each)."""
    return 1 if i <= 256 else 2 if i <= 512 else 4 if i <= 1024 else 8


def unit_lanes(q, l8):
    """Lanes q, q + 8, q + 16, q + 24 of a part that hold values (lane l < l8)."""
    return min(4, (l8 - q + 7) // 8) if l8 > q else 0


def regroup_w2(W2):
    """W2 [E, H, I] -> W2F [E, H * I]: per expert, per part p (of unit_parts(I) parts of Lp values),
    per lane class q = 0..7, the rows [H][8 nl] of lanes q, q + 8, q + 16, q + 24 that hold values
    (lane l holds the part's values [8 l, 8 l + 8)), lanes in that order. The same values as W2,
    in the order one expert unit streams them."""
    E, H, I = W2.shape
    kp = unit_parts(I)
    lp = I // kp
    l8 = lp // 8
    assert lp % 8 == 0 and l8 <= 32, (I, kp)
    x = W2.reshape(E, H, kp, l8, 8)
    if l8 < 32:
        x = torch.cat([x, x.new_zeros(E, H, kp, 32 - l8, 8)], dim=3)
    x = x.reshape(E, H, kp, 4, 8, 8).permute(0, 2, 4, 1, 3, 5)     # [E, kp, q, H, j, k]: lane q + 8 j
    pieces = [x[:, :, q, :, :unit_lanes(q, l8), :].reshape(E, kp, H * 8 * unit_lanes(q, l8))
              for q in range(8) if unit_lanes(q, l8)]
    return torch.cat(pieces, dim=2).reshape(E, H * I).contiguous()


E4M3_MAX = 448.0


def quantize_e4m3(w, groups=1):
    """Weight-only FP8 (the reference's D26): w [E, R, K] BF16 -> (q [E, R, K] uint8 E4M3 codes,
    scale [E, groups] float32). Rows r with r mod groups = g form one tensor with one scale,
    amax / 448 (1 for an all-zero tensor); q = e4m3(w / scale), the quotient in FP32, rounded to
    the nearest E4M3 value (ties to even), |w / scale| <= 448 by construction. groups = 2 for the
    interleaved gate/up rows of W13 (gate and up are separate tensors in a checkpoint)."""
    E, R, K = w.shape
    assert R % groups == 0
    wf = w.float().reshape(E, R // groups, groups, K)
    amax = wf.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (wf / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(E, R, K).contiguous(), scale.contiguous()


def fp8_experts(W13, W2):
    """The expert units' FP8 tensors of one layer: (W13q [E, 2I, H] uint8, s13 [E, 2], W2Fq
    [E, H * I] uint8 regrouped as regroup_w2 orders it, s2 [E])."""
    W13q, s13 = quantize_e4m3(W13, 2)
    W2q, s2 = quantize_e4m3(W2, 1)
    return W13q, s13, regroup_w2(W2q), s2.reshape(-1).contiguous()


def pack_attention(d: Dims, get):
    """The attention and norm tensors of one layer; get(suffix) -> the layer's tensor."""
    w_uk, w_uv = split_uk_uv(d, get("self_attn.kv_b_proj.weight"))
    out = {"w_norm1": get("input_layernorm.weight").contiguous(),
           "w_norm2": get("post_attention_layernorm.weight").contiguous(),
           "W_qkva": pack_qkva(get("self_attn.q_proj.weight"), get("self_attn.kv_a_proj_with_mqa.weight")),
           "w_kv_norm": get("self_attn.kv_a_layernorm.weight").contiguous(),
           "W_ukT": transpose_uk(w_uk), "W_uv": w_uv.contiguous(),
           "W_o": get("self_attn.o_proj.weight").contiguous()}
    if tuple(out["W_qkva"].shape) != (d.QKVA_OUT, d.H) or tuple(out["W_o"].shape) != (d.H, d.NH * d.D_V):
        raise ValueError(f"attention shapes: W_qkva {tuple(out['W_qkva'].shape)}, W_o {tuple(out['W_o'].shape)}")
    return out


def pack_layer(d: Dims, l, get):
    """Every packed tensor of layer l (without the _{l} suffix); get(suffix) -> the layer's tensor,
    or a dict {suffix: tensor}."""
    if isinstance(get, dict):
        get = get.__getitem__
    out = pack_attention(d, get)
    mlp = lambda name: get(f"mlp.{name}.weight")  # noqa: E731
    if l == 0:
        out.update(pack_dense_mlp(d, mlp("gate_proj"), mlp("up_proj"), mlp("down_proj")))
    else:
        experts = [tuple(mlp(f"experts.{e}.{p}") for p in ("gate_proj", "up_proj", "down_proj")) for e in range(d.E)]
        shared = tuple(mlp(f"shared_experts.{p}") for p in ("gate_proj", "up_proj", "down_proj"))
        out.update(pack_moe(d, mlp("gate"), experts, shared))
    return out


def _pack_model(d: Dims, fetch, layers, head):
    """The packed dict of a model whose tensors fetch(name) returns by checkpoint name."""
    packed = {"W_embed": fetch("model.embed_tokens.weight").contiguous()}
    if head:
        packed["W_lm"] = fetch("lm_head.weight").contiguous()
        packed["w_final_norm"] = fetch("model.norm.weight").contiguous()
    for l in range(d.L if layers is None else layers):
        prefix = f"model.layers.{l}."
        packed.update({f"{k}_{l}": v for k, v in pack_layer(d, l, lambda s: fetch(prefix + s)).items()})
    return packed


def pack_state_dict(d: Dims, sd, layers=None, head=True):
    """An HF state dict (names as the checkpoint's) -> the packed dict, keys suffixed `_{l}`."""
    return _pack_model(d, sd.__getitem__, layers, head)


# ----------------------------------------------------------------------------
# byte accounting (from dims only)


def layer_bytes(d: Dims, l, bf16=2):
    """Bytes of one layer's packed weights."""
    attn = 2 * d.H + d.QKVA_OUT * d.H + d.D_C + d.KVB_OUT * d.D_C + d.H * d.NH * d.D_V
    if l == 0:
        return (attn + 3 * d.I_DENSE * d.H) * bf16
    return (attn + d.E * d.H + d.E_TOTAL * 3 * d.I_MOE * d.H) * bf16


def packed_bytes(d: Dims, bf16=2):
    """Every packed byte (the checkpoint's 31,412,968,448 at REAL_DIMS: nothing is padded)."""
    return 2 * d.V * d.H * bf16 + d.H * bf16 + sum(layer_bytes(d, l, bf16) for l in range(d.L))


def active_bytes_per_token(d: Dims, ctx=1024, layers=None, head=True, bf16=2, expert_bytes=None):
    """Algorithmic HBM bytes of one decode token, counted as the reference's roofline counts
    them (docs/deepseek-v2-lite/sources/roofline.py; 07-roofline.md:30-55): every attention and
    dense-MLP weight matrix, the router, the shared and TOPK routed experts of each MoE layer,
    lm_head, and `ctx` latent-cache rows per layer. Norm weights and the embedding row (under
    0.01%) are not counted. At REAL_DIMS, ctx 1024: 4,934,467,584 B. expert_bytes: bytes per
    expert weight (1 for the FP8 experts, whose scales are 12 bytes an expert; default bf16)."""
    layers = d.L if layers is None else layers
    eb = bf16 if expert_bytes is None else expert_bytes
    attn = d.Q_OUT * d.H + d.KVA_OUT * d.H + d.KVB_OUT * d.D_C + d.H * d.NH * d.D_V
    total = 0
    for l in range(layers):
        total += (attn + ctx * (d.D_C + d.D_R)) * bf16
        if l == 0:
            total += 3 * d.I_DENSE * d.H * bf16
        else:
            total += d.E * d.H * bf16 + d.N_SLOTS * 3 * d.I_MOE * d.H * eb
    if head:
        total += d.V * d.H * bf16
    return total


def routed_bytes_per_token(d: Dims, layers=None, bf16=2):
    """The routed experts' share of active_bytes_per_token: TOPK experts per MoE layer."""
    layers = d.L if layers is None else layers
    return max(0, layers - 1) * d.TOPK * 3 * d.I_MOE * d.H * bf16


def slot_bytes_per_token(d: Dims, layers=None, bf16=2):
    """One expert slot's weights over a token's MoE layers (expert parallelism deals the N_SLOTS
    slots among the ranks)."""
    layers = d.L if layers is None else layers
    return max(0, layers - 1) * 3 * d.I_MOE * d.H * bf16


def moe_layer_bytes(d: Dims, ctx=1025, bf16=2):
    """Algorithmic bytes of one MoE layer's decode step (config 0): attention weights, the three
    norm vectors, the router, N_SLOTS experts and `ctx` cache rows. 167,389,312 B at REAL_DIMS
    and ctx 1025 (position 1024)."""
    attn = d.Q_OUT * d.H + d.KVA_OUT * d.H + d.KVB_OUT * d.D_C + d.H * d.NH * d.D_V
    norms = 2 * d.H + d.D_C
    return (attn + norms + d.E * d.H + d.N_SLOTS * 3 * d.I_MOE * d.H + ctx * (d.D_C + d.D_R)) * bf16


# ----------------------------------------------------------------------------
# synthetic weights


def synthetic_packed(d: Dims, layers=None, head=True, seed=0, device="cuda", std=0.02,
                     norm_weight=1.0, random_norms=False):
    """Seeded random weights in the packed layout: BF16 ~N(0, std) drawn in FP32 from one
    torch.Generator on `device` and rounded, in the fixed order of this function; RMSNorm weights
    `norm_weight` (1.0 in the benchmark configs) or, with random_norms, 1 + 0.5 N(0,1) so a
    mixed-up norm weight shows in the parity tests. The same seed on the same device type gives
    the same bytes; the values depend on the device type (CPU and CUDA generators differ)."""
    layers = d.L if layers is None else layers
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)

    def nw(n):
        if random_norms:
            return (1.0 + 0.5 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)
        return torch.full((n,), norm_weight, dtype=torch.bfloat16, device=device)

    packed = {"W_embed": w(d.V, d.H)}
    for l in range(layers):
        packed[f"w_norm1_{l}"] = nw(d.H)
        packed[f"w_norm2_{l}"] = nw(d.H)
        packed[f"W_qkva_{l}"] = w(d.QKVA_OUT, d.H)
        packed[f"w_kv_norm_{l}"] = nw(d.D_C)
        packed[f"W_ukT_{l}"] = w(d.NH, d.D_C, d.D_N)
        packed[f"W_uv_{l}"] = w(d.NH, d.D_V, d.D_C)
        packed[f"W_o_{l}"] = w(d.H, d.NH * d.D_V)
        if l == 0:
            packed["W_gu_0"] = w(2 * d.I_DENSE, d.H)
            packed["W_down_0"] = w(d.H, d.I_DENSE)
        else:
            packed[f"W_gate_{l}"] = w(d.E, d.H)
            packed[f"W13_{l}"] = w(d.E_TOTAL, 2 * d.I_MOE, d.H)
            packed[f"W2_{l}"] = w(d.E_TOTAL, d.H, d.I_MOE)
    if head:
        packed["w_final_norm"] = nw(d.H)
        packed["W_lm"] = w(d.V, d.H)
    return packed


# ----------------------------------------------------------------------------
# the checkpoint reader (no checkpoint is present in this build's environment; the tests write a
# small one)


def layer_names(d: Dims, l):
    """The checkpoint tensor names of layer l (the HF DeepseekV2 naming)."""
    attn = ("input_layernorm", "post_attention_layernorm", "self_attn.q_proj", "self_attn.kv_a_proj_with_mqa",
            "self_attn.kv_a_layernorm", "self_attn.kv_b_proj", "self_attn.o_proj")
    mlp = ["mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"] if l == 0 else (
        ["mlp.gate"] + [f"mlp.shared_experts.{p}" for p in ("gate_proj", "up_proj", "down_proj")]
        + [f"mlp.experts.{e}.{p}" for e in range(d.E) for p in ("gate_proj", "up_proj", "down_proj")])
    return [f"model.layers.{l}.{n}.weight" for n in list(attn) + mlp]


_ST_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


class SafetensorsDir:
    """A safetensors checkpoint directory read through memory maps of its shards.

    The format: each shard is an 8-byte little-endian header length, a JSON header mapping tensor
    names to {dtype, shape, data_offsets: [begin, end)} relative to the end of the header, then the
    data. model.safetensors.index.json (when present) maps every tensor name to its shard. A tensor
    is copied out of the map straight to `device`; only BF16 weights are accepted."""

    def __init__(self, model_dir, device="cpu"):
        self.dir = Path(model_dir)
        self.device = device
        self._open = {}
        index = self.dir / "model.safetensors.index.json"
        if index.exists():
            self.where = dict(json.loads(index.read_text())["weight_map"])
        else:
            self.where = {n: "model.safetensors" for n in self._shard("model.safetensors")[1]}

    def _shard(self, fname):
        """(memory map, header, first data byte) of one shard, opened once."""
        if fname not in self._open:
            import mmap
            with open(self.dir / fname, "rb") as f:
                mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
            n = int.from_bytes(mm[:8], "little")
            header = json.loads(mm[8:8 + n].decode("utf-8"))
            header.pop("__metadata__", None)
            self._open[fname] = (mm, header, 8 + n)
        return self._open[fname]

    def names(self):
        return sorted(self.where)

    def tensor(self, name):
        mm, header, base = self._shard(self.where[name])
        h = header[name]
        if h["dtype"] != "BF16":
            raise ValueError(f"{name}: {h['dtype']} weights; the packer takes BF16 checkpoints")
        b0, b1 = h["data_offsets"]
        buf = memoryview(mm)[base + b0:base + b1]
        t = torch.frombuffer(buf, dtype=torch.int16).view(_ST_DTYPES[h["dtype"]]).reshape(h["shape"])
        return t.to(self.device, copy=True)


def load_checkpoint_layer(model_dir, l, d: Dims, device="cpu", reader=None):
    """The raw tensors of layer l, keyed by their suffix after 'model.layers.{l}.'."""
    reader = reader or SafetensorsDir(model_dir, device)
    prefix = f"model.layers.{l}."
    return {n[len(prefix):]: reader.tensor(n) for n in layer_names(d, l)}


def pack_all(model_dir, device="cpu", dims: Dims = None, layers: int = None, head: bool = True):
    """Every packed tensor of a checkpoint directory (config.json + safetensors shards), keyed by
    name with the layer suffix `_{l}`; layers / head restrict it to a truncated graph's needs."""
    model_dir = Path(model_dir)
    d = dims or Dims.from_config(json.loads((model_dir / "config.json").read_text()))
    check_tiling(d)
    packed = _pack_model(d, SafetensorsDir(model_dir, device).tensor, layers, head)
    if head and (layers is None or layers == d.L):
        total = sum(v.numel() * v.element_size() for v in packed.values())
        if total != packed_bytes(d):
            raise ValueError(f"packed {total} bytes, the dims say {packed_bytes(d)}")
    return packed


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-dir", required=True)
    ap.add_argument("--device", default="cpu")
    args = ap.parse_args()
    packed = pack_all(args.model_dir, args.device)
    total = sum(v.numel() * v.element_size() for v in packed.values())
    print(f"packed {len(packed)} tensors, {total} bytes ({total / 2**20:.1f} MiB)")


if __name__ == "__main__":
    main()
