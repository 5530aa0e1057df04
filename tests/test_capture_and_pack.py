"""Host-side inputs of the decode step: the YaRN tables and softmax scale against the reference
model's own modules (fixtures), and the packed-weight layout and byte accounting."""
import json

import numpy as np
import pytest
import torch

from fleet import capture as C
from fleet import pack_weights as P


def u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_yarn_tables_bit_identical_real_shape(golden):
    fx = golden("yarn_real.npz")
    rows = fx["rows"]
    cos, sin = C.rope_tables(64, int(rows.max()) + 1)
    assert np.array_equal(u16(cos[rows]), fx["cos"])
    assert np.array_equal(u16(sin[rows]), fx["sin"])
    inv = C.yarn_inv_freq(64, 10000.0, 40.0, 4096, 32, 1)
    assert np.array_equal(inv.numpy(), fx["inv_freq"])


def test_yarn_tables_bit_identical_tiny(golden):
    fx = golden("hf_tiny.npz")
    s_max = fx["cos"].shape[0]
    cos, sin = C.rope_tables(8, s_max)
    assert np.array_equal(u16(cos), fx["cos"]) and np.array_equal(u16(sin), fx["sin"])


def test_softmax_scale():
    assert C.softmax_scale(128, 64) == 0.1147213867929261       # harness/common.py:21
    assert abs(C.softmax_scale(16, 8) - 0.3244810821936116) < 1e-16


def test_packed_bytes_match_checkpoint():
    assert P.packed_bytes(P.REAL_DIMS) == P.CHECKPOINT_BYTES


def test_roofline_bytes_match_reference():
    # docs/deepseek-v2-lite/07-roofline.md:47-55
    assert P.active_bytes_per_token(P.REAL_DIMS, ctx=1024) == 4_934_467_584
    # docs/design-doc/09-expected-performance.md:34 (one MoE layer at position 1024)
    assert P.moe_layer_bytes(P.REAL_DIMS, ctx=1025) == 167_389_312


def test_pack_state_dict_roundtrip(golden):
    fx = golden("hf_tiny.npz")
    cfg = json.loads(str(fx["config"]))
    d = P.Dims.from_config(cfg)
    sd = {k[2:]: torch.from_numpy(fx[k].astype(np.int16)).view(torch.bfloat16) for k in fx.files if k.startswith("w:")}
    packed = P.pack_state_dict(d, sd)
    kvb = sd["model.layers.1.self_attn.kv_b_proj.weight"].view(d.NH, d.D_N + d.D_V, d.D_C)
    assert torch.equal(packed["W_ukT_1"], kvb[:, :d.D_N].transpose(1, 2))
    assert torch.equal(packed["W_uv_1"], kvb[:, d.D_N:])
    sh = sd["model.layers.2.mlp.shared_experts.gate_proj.weight"]
    assert torch.equal(packed["W13_2"][d.E + 1, 0::2], sh[d.I_MOE:2 * d.I_MOE])
    assert torch.equal(packed["W2_2"][d.E, :, :], sd["model.layers.2.mlp.shared_experts.down_proj.weight"][:, :d.I_MOE])
    assert torch.equal(packed["W13_1"][3, 1::2], sd["model.layers.1.mlp.experts.3.up_proj.weight"])
    assert torch.equal(packed["W_gu_0"][1::2], sd["model.layers.0.mlp.up_proj.weight"])
    g, u = P.deinterleave_gate_up(packed["W13_1"][5])
    assert torch.equal(g, sd["model.layers.1.mlp.experts.5.gate_proj.weight"]) and torch.equal(u, sd["model.layers.1.mlp.experts.5.up_proj.weight"])
    total = sum(v.numel() * v.element_size() for v in packed.values())
    assert total == P.packed_bytes(d)


def test_synthetic_deterministic():
    d = P.Dims(H=64, NH=2, D_N=16, D_R=8, D_V=16, D_C=32, V=256, L=3, I_DENSE=96, I_MOE=32, E=8, TOPK=2, N_SHARED=2)
    a = P.synthetic_packed(d, device="cpu", seed=7)
    b = P.synthetic_packed(d, device="cpu", seed=7)
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)
    assert float(a["W_qkva_1"].float().std()) < 0.03
    assert torch.all(a["w_norm1_0"] == 1.0)
    assert sum(v.numel() * v.element_size() for v in a.values()) == P.packed_bytes(d)


def test_auto_head_group():
    """One attention task per head at 1K context; at long context heads share a task (and its
    streamed cache rows) as long as every CTA still gets a task."""
    from fleet.graph_plan import auto_head_group, build_plan
    assert auto_head_group(16, 9) == 1          # 1K context: 144 tasks
    assert auto_head_group(16, 33) == 2         # 4K: 264 tasks
    assert auto_head_group(16, 65) == 4         # 8K: 260 tasks
    assert auto_head_group(16, 257) == 16       # 32K: 257 tasks
    assert build_plan(s_max=8200, layers=2).head_group == 4
    assert build_plan(s_max=1056, layers=2).head_group == 1


def test_checkpoint_loader_matches_state_dict(golden, tmp_path):
    """The real-checkpoint loader (pack_all over a sharded safetensors directory, the reference's
    fleet/pack_weights.py:275-339 role) gives the same packed tensors as packing the state dict:
    the tiny reference model's weights written as a two-shard HF checkpoint."""
    from safetensors.torch import save_file
    fx = golden("hf_tiny.npz")
    cfg = json.loads(str(fx["config"]))
    d = P.Dims.from_config(cfg)
    sd = {k[2:]: torch.from_numpy(fx[k].astype(np.int16)).view(torch.bfloat16) for k in fx.files if k.startswith("w:")}
    names = sorted(sd)
    shards = {"model-00001-of-00002.safetensors": names[: len(names) // 2],
              "model-00002-of-00002.safetensors": names[len(names) // 2:]}
    weight_map = {}
    for fname, keys in shards.items():
        save_file({k: sd[k].contiguous() for k in keys}, str(tmp_path / fname))
        weight_map.update({k: fname for k in keys})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    got = P.pack_all(tmp_path)
    want = P.pack_state_dict(d, sd)
    assert got.keys() == want.keys()
    for k in want:
        assert got[k].dtype == torch.bfloat16 and torch.equal(got[k], want[k]), k


def test_checkpoint_reader_single_file_and_dtype(golden, tmp_path):
    """The reader without an index (one model.safetensors), and its refusal of non-BF16 weights."""
    from safetensors.torch import save_file
    fx = golden("hf_tiny.npz")
    cfg = json.loads(str(fx["config"]))
    d = P.Dims.from_config(cfg)
    sd = {k[2:]: torch.from_numpy(fx[k].astype(np.int16)).view(torch.bfloat16) for k in fx.files if k.startswith("w:")}
    save_file({k: v.contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    got, want = P.pack_all(tmp_path), P.pack_state_dict(d, sd)
    assert got.keys() == want.keys() and all(torch.equal(got[k], want[k]) for k in want)
    rd = P.SafetensorsDir(tmp_path)
    assert rd.names() == sorted(sd)
    bad = tmp_path / "f32"
    bad.mkdir()
    save_file({"x": torch.zeros(4)}, str(bad / "model.safetensors"))
    with pytest.raises(ValueError):
        P.SafetensorsDir(bad).tensor("x")


def test_router_biases_zipf_and_uniform():
    """Config 3's injected routing: seeded, one bias per MoE layer, Zipf-shaped or zero."""
    d = P.Dims(H=64, NH=2, D_N=16, D_R=8, D_V=16, D_C=32, V=256, L=4, I_DENSE=96, I_MOE=32, E=64, TOPK=6, N_SHARED=2)
    z = C.router_biases(d, 4, "zipf", device="cpu")
    assert sorted(z) == ["router_bias_1", "router_bias_2", "router_bias_3"]
    b = z["router_bias_1"].numpy()
    assert b.dtype == np.float32 and b.shape == (64,)
    assert np.isclose(b.max(), 3.0) and np.allclose(np.sort(b)[::-1], 3.0 / np.arange(1, 65) ** 1.2, rtol=1e-6)
    assert np.array_equal(C.router_biases(d, 4, "zipf", device="cpu")["router_bias_2"].numpy(),
                          z["router_bias_2"].numpy())
    assert not np.array_equal(z["router_bias_1"].numpy(), z["router_bias_2"].numpy())
    assert all(float(t.abs().sum()) == 0.0 for t in C.router_biases(d, 4, "uniform", device="cpu").values())
