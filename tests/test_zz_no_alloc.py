"""The allocation-free MLA decode entry point (mk_mla_decode_noalloc) against the existing one.

Some callers cannot call cudaMalloc at the point where they run attention: an engine that has
reserved all of HBM for its own memory pool, code running while its own allocator holds a lock,
or a decode loop that cannot afford the synchronisation cudaMalloc/cudaFree bring. For them the
library keeps the split-KV partials in a static device array instead of a caller or library
allocation. These tests call that entry point through the C ABI and check each result bit for bit
(this suite's tolerance for this path is exact equality):

* twice in a row, with different inputs and positions, against the persistent kernel's
  MLA_ATTEND + MLA_MERGE_UV operators on the same inputs;
* over many seeds and positions at the model's shape (16 heads, d_c 512), so that a summation
  order that differs from the specified one (it changes about one BF16 output in 10^4) cannot
  pass by chance: about 98,000 outputs are compared;
* at a small shape (4 heads, d_c 64, d_r 16, d_v 32: one rope column per lane, a one-part row
  dot, fewer than 16 heads) with a short last split, against the CPU oracle and the persistent
  kernel.

They must pass on their own in a fresh process and after the rest of the suite; the file is
collected last so that a run that stops at the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, s_max, nh=16, d_r=64, d_c=512, d_v=128):
    g = torch.Generator(device=DEV).manual_seed(seed)
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=DEV) * std).to(torch.bfloat16)  # noqa: E731
    return dict(ql_nope=bf(nh, d_c), q_pe=bf(nh, d_r), c_kv=bf(s_max, d_c), k_pe=bf(s_max, d_r),
                w_uv=bf(nh, d_v, d_c, std=0.05))


class _Existing:
    """The same computation through the persistent kernel (its partials are an allocated tensor)."""

    def __init__(self, mk, B, x, split, scale):
        from fleet.graph_plan import partials_row
        nh, d_c = x["ql_nope"].shape
        s_max = x["c_kv"].shape[0]
        n_splits = -(-s_max // split)
        self.partials = torch.zeros(n_splits, nh, partials_row(d_c), dtype=torch.float32, device=DEV)
        self.attn = torch.zeros(nh * x["w_uv"].shape[1], dtype=torch.bfloat16, device=DEV)
        self.k = mk.MegaKernel(0)
        self.k.add(B.mla_attend_layer(mk, None, x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], self.partials, scale,
                                      split, n_splits, 1))
        self.k.add(B.mla_merge_uv_layer(mk, None, self.partials, x["w_uv"], self.attn, split, n_splits))
        self.k.finalize()

    def __call__(self, pos):
        self.k.launch(1, pos - 1)
        assert self.k.status()["error"] == 0
        return self.attn.clone()

    def close(self):
        self.k.close()


def _noalloc(mk, x, pos, split, scale):
    got = torch.full((x["ql_nope"].shape[0] * x["w_uv"].shape[1],), 7.0, dtype=torch.bfloat16, device=DEV)
    mk.mla_decode_noalloc(x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], x["w_uv"], got, pos, split, scale)
    torch.cuda.synchronize()
    return got


def _same(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_noalloc_matches_persistent_kernel_twice():
    from fleet import build_graph as B
    from fleet import mk
    from fleet.capture import softmax_scale
    scale = softmax_scale(128, 64)
    split = 64
    for seed, s_max, pos in ((1, 1056, 1024), (2, 2048, 1700)):
        x = _inputs(seed, s_max)
        ex = _Existing(mk, B, x, split, scale)
        want = ex(pos)
        ex.close()
        got = _noalloc(mk, x, pos, split, scale)
        assert _same(got, want), f"seed {seed}: differs from the persistent kernel"


def test_noalloc_matches_persistent_kernel_many_positions():
    from fleet import build_graph as B
    from fleet import mk
    from fleet.capture import softmax_scale
    scale = softmax_scale(128, 64)
    n = 0
    for seed, split in ((11, 64), (12, 32), (13, 128), (14, 64)):
        x = _inputs(seed, 2048)
        ex = _Existing(mk, B, x, split, scale)
        for pos in (0, 31, 63, 64, 200, 511, 700, 1023, 1024, 1500, 1777, 2047):
            if -(-(pos + 1) // split) > 64:
                continue
            want = ex(pos)
            got = _noalloc(mk, x, pos, split, scale)
            assert _same(got, want), f"seed {seed}, split {split}, pos {pos}: differs from the persistent kernel"
            n += got.numel()
        ex.close()
    assert n >= 90_000, n


def test_noalloc_small_shape_matches_oracle_and_kernel():
    from fleet import build_graph as B
    from fleet import mk
    from oracle import numpy_ref as R
    nh, d_r, d_c, d_v, split, scale = 4, 16, 64, 32, 24, 0.17
    np32 = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    for seed, pos in ((21, 100), (22, 47), (23, 250)):        # last splits of 5, 0 (full), 11 rows
        x = _inputs(seed, 256, nh=nh, d_r=d_r, d_c=d_c, d_v=d_v)
        got = _noalloc(mk, x, pos, split, scale)
        ex = _Existing(mk, B, x, split, scale)
        want = ex(pos)
        ex.close()
        assert _same(got, want), f"seed {seed}, pos {pos}: differs from the persistent kernel"
        partials = R.mla_attend(np32(x["ql_nope"]), np32(x["q_pe"]), np32(x["c_kv"]), np32(x["k_pe"]), pos, scale,
                                split=split)
        ref = R.mla_merge_uv(partials, np32(x["w_uv"]), pos, split=split)
        assert np.array_equal(np32(got), ref), f"seed {seed}, pos {pos}: differs from the oracle"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from fleet import mk
    x = _inputs(3, 65 * 64)                  # rows for the whole request, though it must be refused
    out = torch.zeros(16 * 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(mk.MkError):          # 65 splits of 64 rows: more than the static array holds
        mk.mla_decode_noalloc(x["ql_nope"], x["q_pe"], x["c_kv"], x["k_pe"], x["w_uv"], out, 65 * 64 - 1, 64, 0.1)
