"""The decode step's non-weight inputs: the YaRN RoPE tables, the softmax scale and the latent
cache the prefill leaves behind.

The reference reads these from the HF run's ``ref_cache.safetensors`` (harness/run_fleet.py:533-539,
written by harness/run_reference.py:433-441). Here they are computed on the host:

* ``rope_tables`` restates DeepseekV2YarnRotaryEmbedding (modeling_deepseek.py:262-330): the
  inverse frequencies blended between interpolated and extrapolated by the linear ramp between the
  correction dims of beta_fast/beta_slow, FP32 ``outer(t, inv_freq)``, ``cat(f, f)``, cos/sin
  times the mscale ratio, then BF16. It runs the same torch FP32 CPU operations in the same order,
  so the tables are bit-identical to the model's (tests/test_capture.py against a fixture the
  reference's module produced).
* ``softmax_scale``: q_head_dim^-0.5 times yarn_get_mscale(factor, mscale_all_dim)^2
  (modeling_deepseek.py:745-751); 0.1147213867929261 for DeepSeek-V2-Lite.
* ``synthetic_cache``: the seeded latent rows of the benchmark configs (c_kv and k_pe ~N(0,1)
  BF16) standing in for a prefill.
"""
import math

import torch

# DeepSeek-V2-Lite's rope_scaling (docs/deepseek-v2-lite/sources/config.json)
YARN = dict(base=10000.0, factor=40.0, original_max_position_embeddings=4096, beta_fast=32,
            beta_slow=1, mscale=0.707, mscale_all_dim=0.707)


def yarn_get_mscale(scale=1.0, mscale=1.0):
    if scale <= 1:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


def _correction_dim(num_rotations, dim, base, max_pos):
    return (dim * math.log(max_pos / (num_rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_inv_freq(dim, base, factor, original_max_position_embeddings, beta_fast, beta_slow):
    """FP32 inverse frequencies [dim/2] of the YaRN-scaled rotary embedding."""
    freq_extra = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    freq_inter = 1.0 / (factor * base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    low = max(math.floor(_correction_dim(beta_fast, dim, base, original_max_position_embeddings)), 0)
    high = min(math.ceil(_correction_dim(beta_slow, dim, base, original_max_position_embeddings)), dim - 1)
    if low == high:
        high += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low), 0, 1)
    extra_mask = 1.0 - ramp
    return freq_inter * (1 - extra_mask) + freq_extra * extra_mask


def rope_tables(d_r, s_max, yarn=None, device="cpu"):
    """(cos, sin) [s_max, d_r] BF16 for positions 0..s_max-1."""
    y = dict(YARN if yarn is None else yarn)
    inv_freq = yarn_inv_freq(d_r, y["base"], y["factor"], y["original_max_position_embeddings"],
                             y["beta_fast"], y["beta_slow"])
    t = torch.arange(s_max, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    m = float(yarn_get_mscale(y["factor"], y["mscale"]) / yarn_get_mscale(y["factor"], y["mscale_all_dim"]))
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = (emb.cos() * m).to(torch.bfloat16)
    sin = (emb.sin() * m).to(torch.bfloat16)
    return cos.contiguous().to(device), sin.contiguous().to(device)


def softmax_scale(d_n, d_r, yarn=None):
    y = YARN if yarn is None else yarn
    s = (d_n + d_r) ** -0.5
    if y and y.get("mscale_all_dim"):
        m = yarn_get_mscale(y["factor"], y["mscale_all_dim"])
        s = s * m * m
    return s


def synthetic_cache(dims, layers, s_max, n_past, seed=1, device="cuda"):
    """{c_kv_l [s_max, D_C], k_pe_l [s_max, D_R]} BF16 with rows [0, n_past) ~N(0,1) from one
    torch.Generator (layer by layer, c_kv then k_pe) and the rows the decode will write zeroed."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    cap = {}
    for l in range(layers):
        c = torch.zeros(s_max, dims.D_C, dtype=torch.bfloat16, device=device)
        k = torch.zeros(s_max, dims.D_R, dtype=torch.bfloat16, device=device)
        c[:n_past] = torch.randn(n_past, dims.D_C, generator=g, device=device).to(torch.bfloat16)
        k[:n_past] = torch.randn(n_past, dims.D_R, generator=g, device=device).to(torch.bfloat16)
        cap[f"c_kv_{l}"] = c
        cap[f"k_pe_{l}"] = k
    return cap


def make_capture(dims, layers, s_max, n_past, seed=1, device="cuda", yarn=None):
    """The reference's ``capture`` dict: cos, sin and the per-layer latent cache."""
    cos, sin = rope_tables(dims.D_R, s_max, yarn, device)
    cap = {"cos": cos, "sin": sin}
    cap.update(synthetic_cache(dims, layers, s_max, n_past, seed, device))
    return cap


def router_biases(dims, layers, kind, seed=4, device="cuda", scale=3.0, s_zipf=1.2):
    """Injected router logit biases [E] (FP32) for the MoE layers 1..layers-1, config 3's routing:
    "zipf" ranks the experts by a seeded permutation per layer and adds scale / rank^s_zipf, so the
    top-6 choices skew towards the low ranks; "uniform" adds nothing (every expert equally likely
    under the seeded synthetic weights)."""
    import numpy as np
    import torch

    out = {}
    for l in range(1, layers):
        if kind == "zipf":
            ranks = np.random.default_rng(seed + l).permutation(dims.E) + 1
            b = (scale * (1.0 / ranks.astype(np.float64) ** s_zipf)).astype(np.float32)
        elif kind == "uniform":
            b = np.zeros(dims.E, np.float32)
        else:
            raise ValueError(f"routing kind {kind!r}: uniform or zipf")
        out[f"router_bias_{l}"] = torch.from_numpy(b).to(device)
    return out
