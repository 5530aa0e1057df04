"""The C-ABI library without a GPU: it loads, exports every entry point include/fleet_mk.h declares,
reports its version, and the ctypes structs match the header's layout."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "fleet_mk.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(mk_\w+)\(", text, re.M)))


def test_header_declarations_bound():
    from fleet import mk
    assert declared() == sorted(mk.EXPORTS)


def test_library_exports_every_symbol():
    from fleet import mk
    if not mk.LIB_PATH.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    L = ctypes.CDLL(str(mk.LIB_PATH))
    for name in declared():
        assert hasattr(L, name), name
    assert mk.lib().mk_version() == 1


def test_struct_layout():
    from fleet import mk
    assert ctypes.sizeof(mk.MkOp) == 4 * 4 + 16 * 8 + 16 * 8 + 4 * 8
    assert ctypes.sizeof(mk.MkConfig) == 4 + 4 + 8 + 4 + 7 * 4
    assert ctypes.sizeof(mk.MkStatus) == 6 * 4 + 2 * 8
    assert ctypes.sizeof(mk.MkTraceRecord) == 4 * 4 + 5 * 8


def test_create_without_gpu_fails_cleanly():
    import torch
    from fleet import mk
    if torch.cuda.is_available() or not mk.LIB_PATH.exists():
        pytest.skip("needs the library and no GPU")
    with pytest.raises(mk.MkError):
        mk.MegaKernel(0)


def test_device_constants_match_oracle():
    """The FP32 bit patterns in csrc/detmath.cuh are the oracle's constants."""
    import numpy as np
    from oracle import detmath as D
    src = (ROOT / "fleet-amd-task_b200/csrc/detmath.cuh").read_text()
    pats = {int(v) for v in re.findall(r"__uint_as_float\((\d+)u\)", src)}
    want = {int(np.float32(c).view(np.uint32)) for c in
            [D.LOG2E, D.LN2_HI, D.LN2_LO, D.SQRT2] + D.EXP_C[3:] + D.LOG_C[1:]}
    assert want <= pats, sorted(want - pats)
