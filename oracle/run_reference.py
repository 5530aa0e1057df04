#!/usr/bin/env python3
"""The reference side of a harness comparison for the seeded synthetic configs: what the
reference's harness/run_reference.py writes from the HF model and the real checkpoint
(ref_cache, ref_boundaries_step0, ref_output_ids, ref_route_log, ref_hidden_per_layer_step0,
:339-484), written here from the CPU oracle and the benchmark configs' synthetic weights.

TEST INFRASTRUCTURE: the checker side of tests/test_gpu_harness.py; it runs no kernel of this
repository. The weights are drawn by torch's CUDA generator (fleet.workload), so it needs a CUDA
device to create them; the arithmetic is oracle/model.py's on the host.

    python oracle/run_reference.py --out REF_DIR --layers N [--iters K] [--n-prompt 1024]

The cache stands in for a prefill as in the benchmark (seeded rows 0..n_prompt-2); decode step i
runs at position n_prompt - 1 + i. Files:
    prompt_ids.json, ref_cache.safetensors (cos, sin [S, 64]; c_kv [L, S, 512]; k_pe [L, S, 64]),
    ref_boundaries_step0.safetensors and ref_boundaries_step{K-1}.safetensors (layers 0 and 1 and
    the head), ref_output_ids.json, ref_route_log.json ([step][MoE layer] {"idx", "w", "w_all"}),
    ref_hidden_per_layer_step0.safetensors ({"hidden": [L, H]}).
"""
import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "fleet-amd-task_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

BOUNDARY_LAYERS = (0, 1)


def boundaries(rec, d, layers, pos, token_next, scores=None):
    """The reference's boundary keys from one oracle step's record (BF16 values as BF16 tensors)."""
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)  # noqa: E731
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))  # noqa: E731
    b = {}
    for l in BOUNDARY_LAYERS:
        if l >= layers:
            continue
        b[f"L{l}.B1.norm1"] = bf(rec[f"L{l}.norm1"])
        b[f"L{l}.B2.q"] = bf(rec[f"L{l}.qkva"][:d.Q_OUT])
        b[f"L{l}.B3.c_kv"] = bf(rec[f"L{l}.c_kv"])
        b[f"L{l}.B3.k_pe"] = bf(rec[f"L{l}.k_pe"])
        b[f"L{l}.B4.q_pe"] = bf(rec[f"L{l}.q_pe"])
        b[f"L{l}.B6.attn"] = bf(rec[f"L{l}.attn"])
        b[f"L{l}.B7.x_res_attn"] = bf(rec[f"L{l}.x_res_attn"])
        b[f"L{l}.B13.layer_out"] = bf(rec[f"L{l}.layer_out"])
        if l >= 1:
            mask = rec[f"L{l}.mask"]
            b[f"L{l}.B8.router_logits"] = f32(rec[f"L{l}.router_logits"])
            b[f"L{l}.B9.topk_idx"] = torch.tensor(mask[:d.TOPK].tolist(), dtype=torch.int32)
            b[f"L{l}.B10.topk_w"] = f32(rec[f"L{l}.topk_w"][:d.TOPK])
            for s in range(d.TOPK):
                b[f"L{l}.B11.expert_{int(mask[s])}"] = bf(rec[f"L{l}.out8"][s])
            b[f"L{l}.B12.shared"] = f32(sum(rec[f"L{l}.out8"][s].astype(np.float32) for s in range(d.TOPK, d.N_SLOTS)))
    if "head.logits" in rec:
        b["head.B14.norm"] = bf(rec["head.norm"])
        b["head.B15.logits"] = bf(rec["head.logits"])
        b["head.B16.token"] = torch.tensor([token_next], dtype=torch.int64)
    return b


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--layers", type=int, required=True)
    ap.add_argument("--iters", type=int, default=1)
    ap.add_argument("--n-prompt", type=int, default=1024)
    a = ap.parse_args(argv)
    from safetensors.torch import save_file

    from fleet.capture import softmax_scale
    from fleet.graph_plan import SPLIT
    from fleet.workload import greedy_decode
    from gpu_helpers import DeviceWeightBits, u16
    from oracle import numpy_ref as R
    from oracle.model import OracleModel

    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    w = greedy_decode("cuda:0", n_prompt=a.n_prompt, new_tokens=a.iters, layers=a.layers)
    d = w.dims
    (out / "prompt_ids.json").write_text(json.dumps(w.prompt) + "\n")
    s_max = w.s_max
    cache_t = {"cos": w.capture["cos"].cpu(), "sin": w.capture["sin"].cpu(),
               "c_kv": torch.stack([w.capture[f"c_kv_{l}"].cpu() for l in range(a.layers)]),
               "k_pe": torch.stack([w.capture[f"k_pe_{l}"].cpu() for l in range(a.layers)])}
    save_file({k: v.contiguous() for k, v in cache_t.items()}, str(out / "ref_cache.safetensors"))
    dw = DeviceWeightBits(w.packed, keep_experts=range(d.E, d.E_TOTAL))
    m = OracleModel(d, dw.get, dw.get_expert, softmax_scale=softmax_scale(d.D_N, d.D_R), split=SPLIT,
                    layers=a.layers)
    cache = {k: (u16(v).astype(np.uint32) << 16).view(np.float32) for k, v in w.capture.items()
             if k.startswith(("c_kv_", "k_pe_"))}
    cos, sin = (w.capture[k].float().cpu().numpy() for k in ("cos", "sin"))
    tokens = np.zeros(s_max, np.int64)
    tokens[:w.n_prompt] = w.prompt
    route_log, step_recs = [], {}

    def note(i, rec):
        if i == 0 or i == a.iters - 1:
            step_recs[i] = rec
        entries = []
        for l in range(1, a.layers):
            p = R.softmax_det(rec[f"L{l}.router_logits"])
            entries.append({"idx": rec[f"L{l}.mask"][:d.TOPK].tolist(),
                            "w": [float(x) for x in rec[f"L{l}.topk_w"][:d.TOPK]], "w_all": [float(x) for x in p]})
        route_log.append(entries)

    ids, _, _ = m.generate(tokens, w.first_pos, a.iters, cache, cos, sin, on_step=note)
    for i, rec in step_recs.items():
        save_file(boundaries(rec, d, a.layers, w.first_pos + i, ids[i]), str(out / f"ref_boundaries_step{i}.safetensors"))
    hidden = torch.stack([torch.from_numpy(np.ascontiguousarray(step_recs[0][f"L{l}.layer_out"], np.float32))
                          for l in range(a.layers)]).to(torch.bfloat16)
    save_file({"hidden": hidden}, str(out / "ref_hidden_per_layer_step0.safetensors"))
    (out / "ref_output_ids.json").write_text(json.dumps([int(x) for x in ids]) + "\n")
    (out / "ref_route_log.json").write_text(json.dumps(route_log) + "\n")
    print(json.dumps({"ids": [int(x) for x in ids], "out": str(out)}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
