"""The allocation-free MLA decode entry point (mk_mla_decode_noalloc) against the existing one.

Some callers cannot call cudaMalloc at the point where they run attention: an engine that has
reserved all of HBM for its own memory pool, code running while its own allocator holds a lock,
or a decode loop that cannot afford the synchronisation cudaMalloc/cudaFree bring. For them the
library keeps the split-KV partials in a static device array instead of a caller or library
allocation. This test calls that entry point through the C ABI, twice in a row with different
inputs and positions, and checks each result bit for bit against the persistent kernel's
MLA_ATTEND + MLA_MERGE_UV operators on the same inputs (this suite's tolerance is exact equality).
It must pass on its own in a fresh process and after the rest of the suite, and it is collected
last so that a run that stops at the first failure has already run every other test.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, s_max, nh=16, d_n=128, d_r=64, d_c=512, d_v=128):
    g = torch.Generator(device=DEV).manual_seed(seed)
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=DEV) * std).to(torch.bfloat16)  # noqa: E731
    return dict(ql_nope=bf(nh, d_c), q_pe=bf(nh, d_r), c_kv=bf(s_max, d_c), k_pe=bf(s_max, d_r),
                w_uv=bf(nh, d_v, d_c, std=0.05), d_n=d_n)


def _existing(mk, B, x, pos, split, scale):
    """The same computation through the persistent kernel (its partials are an allocated tensor)."""
    from fleet.graph_plan import partials_row
    nh, d_c = x["ql_nope"].shape
    s_max = x["c_kv"].shape[0]
    n_splits = -(-s_max // split)
    partials = torch.zeros(n_splits, nh, partials_row(d_c), dtype=torch.float32, device=DEV)
    attn = torch.zeros(nh * x["w_uv"].shape[1], dtype=torch.bfloat16, device=DEV)
    k = mk.MegaKernel(0)
    k.add(B.mla_attend_layer(mk, None, x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], partials, scale, split,
                             n_splits, 1))
    k.add(B.mla_merge_uv_layer(mk, None, partials, x["w_uv"], attn, split, n_splits))
    k.finalize()
    k.launch(1, pos - 1)
    assert k.status()["error"] == 0
    k.close()
    return attn


def test_noalloc_matches_persistent_kernel_twice():
    from fleet import build_graph as B
    from fleet import mk
    from fleet.capture import softmax_scale
    scale = softmax_scale(128, 64)
    split = 64
    for seed, s_max, pos in ((1, 1056, 1024), (2, 2048, 1700)):
        x = _inputs(seed, s_max)
        want = _existing(mk, B, x, pos, split, scale)
        got = torch.full_like(want, 7.0)
        mk.mla_decode_noalloc(x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], x["w_uv"], got, pos, split, scale)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"seed {seed}: differs from the kernel"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from fleet import mk
    x = _inputs(3, 65 * 64)                  # rows for the whole request, though it must be refused
    out = torch.zeros(16 * 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(mk.MkError):          # 65 splits of 64 rows: more than the static array holds
        mk.mla_decode_noalloc(x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], x["w_uv"], out, 65 * 64 - 1, 64, 0.1)
