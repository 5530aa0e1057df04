"""The GPU prefill (fleet.build_graph.prefill): the decode graph without the head, teacher-forced
over the prompt in one launch, must leave exactly the cache the oracle's token-by-token prefill
leaves (every row of every layer, bit for bit), and the greedy decode that follows must give the
oracle's ids. DeepSeek-V2-Lite shapes with three layers (dense layer 0, two MoE layers) and a
96-token prompt, so the oracle's prefill runs in seconds; a full launch of 95 iterations."""
import numpy as np
import pytest
import torch

from gpu_helpers import DeviceWeightBits, u16
from oracle.detmath import bf16_bits
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_prefill_then_decode_matches_oracle():
    from fleet import build_graph as B
    from fleet.capture import make_capture, softmax_scale
    from fleet.graph_plan import SPLIT
    from fleet.pack_weights import REAL_DIMS, synthetic_packed
    from fleet.workload import prompt_ids
    d, layers, n_prompt, iters = REAL_DIMS, 3, 96, 4
    s_max = n_prompt + iters
    packed = synthetic_packed(d, layers=layers, head=True, seed=0, device=DEV)
    capture = make_capture(d, layers, s_max, 0, seed=1, device=DEV)      # an empty cache
    for k in capture:
        if k.startswith(("c_kv_", "k_pe_")):
            capture[k].fill_(float("nan"))                               # nothing may read an unwritten row
    prompt = prompt_ids(d, n_prompt)
    meta = B.make_meta(torch, s_max, prompt, n_prompt, device=DEV)
    st = B.prefill(packed, capture, meta, n_prompt, dims=d, s_max=s_max, layers=layers)
    assert st["error"] == 0 and st["generation"] == n_prompt - 1, st
    mpk, host, plan = B.build(packed, capture, meta, dims=d, s_max=s_max, layers=layers, head=True)
    mpk.compile()
    mpk()
    assert mpk.status()["error"] == 0
    ids = meta["tokens"][0, n_prompt:n_prompt + iters].tolist()
    gpu_cache = {k: u16(v) for k, v in capture.items() if k.startswith(("c_kv_", "k_pe_"))}

    dw = DeviceWeightBits(packed, keep_experts=range(d.E, d.E_TOTAL))
    m = OracleModel(d, dw.get, dw.get_expert, softmax_scale=softmax_scale(d.D_N, d.D_R), split=SPLIT, layers=layers)
    cache = {k: np.zeros((s_max, v.shape[1]), np.float32) for k, v in gpu_cache.items()}
    cos, sin = (capture[k].float().cpu().numpy() for k in ("cos", "sin"))
    tokens = np.zeros(s_max, np.int64)
    tokens[:n_prompt] = prompt
    for pos in range(n_prompt - 1):                  # the reference's prefill, one token at a time
        m.step(int(tokens[pos]), pos, cache, cos, sin)
    for k, v in gpu_cache.items():
        bad = np.nonzero(v[:n_prompt - 1] != bf16_bits(cache[k][:n_prompt - 1]))[0]
        assert bad.size == 0, f"{k}: prefill rows {bad[:5]} differ"
    want, _, _ = m.generate(tokens, n_prompt - 1, iters, cache, cos, sin)
    assert ids == want, (ids, want)
    for k, v in gpu_cache.items():
        assert np.array_equal(v[:s_max - 1], bf16_bits(cache[k][:s_max - 1])), k
