#!/usr/bin/env python3
"""Pack DeepSeek-V2-Lite-shaped weights into the tensors the B200 decode graph attaches.

Drop-in for the reference's fleet/pack_weights.py (same entry points: ``Dims``, ``REAL_DIMS``,
``pack_all(model_dir, device, dims, layers, head)``, the pure ``pack_*`` functions and the
safetensors loader), with the B200 layout:

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
# pure packing functions


def pack_qkva(w_q, w_kva):
    """[Q_OUT + KVA_OUT, H]: q rows (head-major, nope then pe), then c, then k_pe_raw."""
    assert w_q.shape[1] == w_kva.shape[1]
    return torch.cat([w_q, w_kva], dim=0)


def split_uk_uv(d: Dims, w_kvb, contiguous=False):
    """kv_b_proj [NH*(D_N+D_V), D_C] -> W_uk [NH, D_N, D_C], W_uv [NH, D_V, D_C] (views unless
    contiguous). Per head h: k_nope[h] = W_uk[h] @ c, v[h] = W_uv[h] @ c."""
    assert w_kvb.shape == (d.KVB_OUT, d.D_C), w_kvb.shape
    v = w_kvb.view(d.NH, d.D_N + d.D_V, d.D_C)
    w_uk, w_uv = v[:, :d.D_N], v[:, d.D_N:]
    if contiguous:
        w_uk, w_uv = w_uk.contiguous(), w_uv.contiguous()
    return w_uk, w_uv


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
    """W13 [E_TOTAL, 2*I_MOE, H] (gate and up rows interleaved) and W2 [E_TOTAL, H, I_MOE], with the
    shared MLP as N_SHARED extra experts: expert E + s holds rows [s*I_MOE, (s+1)*I_MOE) of the
    shared gate/up and the same column range of the shared down (the reference's D6 layout)."""
    assert w_gate_router.shape == (d.E, d.H)
    assert len(experts) == d.E
    sg, su, sd = shared
    assert sg.shape == (d.I_SHARED, d.H) and su.shape == (d.I_SHARED, d.H)
    assert sd.shape == (d.H, d.I_SHARED)
    w13 = torch.empty(d.E_TOTAL, 2 * d.I_MOE, d.H, dtype=sg.dtype, device=sg.device)
    w2 = torch.empty(d.E_TOTAL, d.H, d.I_MOE, dtype=sg.dtype, device=sg.device)
    for e, (g, u, dn) in enumerate(experts):
        assert g.shape == (d.I_MOE, d.H) and u.shape == (d.I_MOE, d.H) and dn.shape == (d.H, d.I_MOE)
        w13[e] = interleave_gate_up(g, u)
        w2[e] = dn
    for s in range(d.N_SHARED):
        e = d.E + s
        rows = slice(s * d.I_MOE, (s + 1) * d.I_MOE)
        w13[e] = interleave_gate_up(sg[rows], su[rows])
        w2[e] = sd[:, rows]
    return {"W_gate": w_gate_router.contiguous(), "W13": w13, "W2": w2}


def pack_attention(d: Dims, lw):
    """Attention and norm tensors of one layer from a dict keyed by HF suffixes."""
    w_uk, w_uv = split_uk_uv(d, lw["self_attn.kv_b_proj.weight"], contiguous=True)
    out = {
        "w_norm1": lw["input_layernorm.weight"].contiguous(),
        "w_norm2": lw["post_attention_layernorm.weight"].contiguous(),
        "W_qkva": pack_qkva(lw["self_attn.q_proj.weight"], lw["self_attn.kv_a_proj_with_mqa.weight"]),
        "w_kv_norm": lw["self_attn.kv_a_layernorm.weight"].contiguous(),
        "W_ukT": transpose_uk(w_uk),
        "W_uv": w_uv,
        "W_o": lw["self_attn.o_proj.weight"].contiguous(),
    }
    assert out["W_qkva"].shape == (d.QKVA_OUT, d.H)
    assert out["W_o"].shape == (d.H, d.NH * d.D_V)
    return out


def pack_layer(d: Dims, l, lw):
    out = pack_attention(d, lw)
    if l == 0:
        out.update(pack_dense_mlp(d, lw["mlp.gate_proj.weight"], lw["mlp.up_proj.weight"],
                                  lw["mlp.down_proj.weight"]))
    else:
        experts = [(lw[f"mlp.experts.{e}.gate_proj.weight"], lw[f"mlp.experts.{e}.up_proj.weight"],
                    lw[f"mlp.experts.{e}.down_proj.weight"]) for e in range(d.E)]
        shared = (lw["mlp.shared_experts.gate_proj.weight"], lw["mlp.shared_experts.up_proj.weight"],
                  lw["mlp.shared_experts.down_proj.weight"])
        out.update(pack_moe(d, lw["mlp.gate.weight"], experts, shared))
    return out


def pack_state_dict(d: Dims, sd, layers=None, head=True):
    """An HF state dict (names as the checkpoint's) -> the packed dict, keys suffixed `_{l}`."""
    packed = {"W_embed": sd["model.embed_tokens.weight"].contiguous()}
    if head:
        packed["W_lm"] = sd["lm_head.weight"].contiguous()
        packed["w_final_norm"] = sd["model.norm.weight"].contiguous()
    for l in range(layers if layers is not None else d.L):
        p = f"model.layers.{l}."
        lw = {n[len(p):]: sd[n] for n in layer_names(d, l)}
        for k, v in pack_layer(d, l, lw).items():
            packed[f"{k}_{l}"] = v
    return packed


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


def active_bytes_per_token(d: Dims, ctx=1024, layers=None, head=True, bf16=2):
    """Algorithmic HBM bytes of one decode token, counted as the reference's roofline counts
    them (docs/deepseek-v2-lite/sources/roofline.py; 07-roofline.md:30-55): every attention and
    dense-MLP weight matrix, the router, the shared and TOPK routed experts of each MoE layer,
    lm_head, and `ctx` latent-cache rows per layer. Norm weights and the embedding row (under
    0.01%) are not counted. At REAL_DIMS, ctx 1024: 4,934,467,584 B."""
    layers = d.L if layers is None else layers
    attn = d.Q_OUT * d.H + d.KVA_OUT * d.H + d.KVB_OUT * d.D_C + d.H * d.NH * d.D_V
    total = 0
    for l in range(layers):
        total += attn + ctx * (d.D_C + d.D_R)
        if l == 0:
            total += 3 * d.I_DENSE * d.H
        else:
            total += d.E * d.H + d.N_SLOTS * 3 * d.I_MOE * d.H
    if head:
        total += d.V * d.H
    return total * bf16


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
# loader (needs a checkpoint; none is present in this build's environment)


def layer_names(d: Dims, l):
    p = f"model.layers.{l}."
    names = [p + s for s in (
        "input_layernorm.weight", "post_attention_layernorm.weight",
        "self_attn.q_proj.weight", "self_attn.kv_a_proj_with_mqa.weight",
        "self_attn.kv_a_layernorm.weight", "self_attn.kv_b_proj.weight",
        "self_attn.o_proj.weight")]
    if l == 0:
        names += [p + f"mlp.{s}.weight" for s in ("gate_proj", "up_proj", "down_proj")]
    else:
        names.append(p + "mlp.gate.weight")
        names += [p + f"mlp.shared_experts.{s}.weight" for s in ("gate_proj", "up_proj", "down_proj")]
        for e in range(d.E):
            names += [p + f"mlp.experts.{e}.{s}.weight" for s in ("gate_proj", "up_proj", "down_proj")]
    return names


class Shards:
    """Lazy reader of a safetensors checkpoint by tensor name (model.safetensors.index.json)."""

    def __init__(self, model_dir, device):
        from safetensors import safe_open

        self.dir = Path(model_dir)
        self.map = json.loads((self.dir / "model.safetensors.index.json").read_text())["weight_map"]
        self.device = device
        self.open = {}
        self._safe_open = safe_open

    def get(self, name):
        shard = self.map[name]
        if shard not in self.open:
            self.open[shard] = self._safe_open(str(self.dir / shard), framework="pt", device=str(self.device))
        t = self.open[shard].get_tensor(name)
        assert t.dtype == torch.bfloat16, (name, t.dtype)
        return t


def load_checkpoint_layer(model_dir, l, d: Dims, device="cpu", shards=None):
    shards = shards or Shards(model_dir, device)
    p = f"model.layers.{l}."
    return {n[len(p):]: shards.get(n) for n in layer_names(d, l)}


def pack_all(model_dir, device="cpu", dims: Dims = None, layers: int = None, head: bool = True):
    """Every packed tensor of a real checkpoint, keyed by name with the layer suffix `_{l}`."""
    model_dir = Path(model_dir)
    if dims is None:
        dims = Dims.from_config(json.loads((model_dir / "config.json").read_text()))
    check_tiling(dims)
    shards = Shards(model_dir, device)
    packed = {"W_embed": shards.get("model.embed_tokens.weight")}
    if head:
        packed["W_lm"] = shards.get("lm_head.weight")
        packed["w_final_norm"] = shards.get("model.norm.weight")
    for l in range(layers if layers is not None else dims.L):
        lw = load_checkpoint_layer(model_dir, l, dims, device, shards)
        for k, v in pack_layer(dims, l, lw).items():
            packed[f"{k}_{l}"] = v
    total = sum(v.numel() * v.element_size() for v in packed.values())
    if head and (layers is None or layers == dims.L):
        assert total == packed_bytes(dims), (total, packed_bytes(dims))
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
