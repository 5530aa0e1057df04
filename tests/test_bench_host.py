"""Host-side pieces of bench.py that need no GPU: the roofline arithmetic across contexts and the
per-operator trace summary over synthetic stamps."""
import io
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from fleet.pack_weights import REAL_DIMS as D, active_bytes_per_token  # noqa: E402


def test_roofline_counts_the_cache_at_the_timed_context():
    r1 = bench.roofline(D, 1.8, 1027, 6450.6, "measured")
    r8 = bench.roofline(D, 2.55, 8195, 6450.6, "measured")
    # one more cached row costs every layer's latent row (512 + 64 BF16 values)
    assert r8["algorithmic_bytes"] - r1["algorithmic_bytes"] == D.L * (8195 - 1027) * (D.D_C + D.D_R) * 2
    assert r1["algorithmic_bytes"] == active_bytes_per_token(D, ctx=1027)
    assert abs(r1["frac"] - r1["achieved"] / 6450.6) < 1e-3


class _Call:
    def __init__(self, label):
        self.label = label


class _Plan:
    def __init__(self, labels):
        self.calls = [_Call(x) for x in labels]


class _Kernel:
    def __init__(self, recs):
        self.recs = recs

    def trace(self):
        return self.recs


class _Mpk:
    def __init__(self, recs):
        self.kernel = _Kernel(recs)


def test_trace_summary_critical_path():
    labels = ["prologue.embed"] + [f"L{l}.{k}" for l in range(5) for k in ("qkva", "mla_attend")] + ["head.lm_head"]
    recs, t = [], 0
    for op, lab in enumerate(labels):
        dur = 3000 if lab.endswith("mla_attend") else 1000          # ns
        for task in range(2):                                          # two tasks on two CTAs
            recs.append((op, task, task, 0, t, t + dur, t + 100, t + dur - 200, 0))
        t += dur
    out = io.StringIO()
    bench.trace_summary(_Mpk(recs), _Plan(labels), out=out)
    text = out.getvalue()
    assert "L2.mla_attend" in text                                    # the middle layer's operators
    line = [x for x in text.splitlines() if x.strip().startswith("mla_attend")][0]
    assert abs(float(line.split()[-1]) - 3.0) < 1e-6                   # its critical-path share, µs
    assert "per layer         4.00" in text
