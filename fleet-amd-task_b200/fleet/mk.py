"""ctypes binding of the sm_100a decode library (include/fleet_mk.h, lib/libfleetmk.so).

This is the thin layer between the reference-shaped Python surface (fleet/build_graph.py,
harness/run_fleet.py) and the CUDA runtime: plain C structs and device pointers; PyTorch only
allocates the tensors whose addresses go in. There is no fallback: if the library is missing or
the device is not a B200, the calls raise.
"""
import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("FLEET_MK_LIB", PKG / "lib" / "libfleetmk.so"))

MK_OK, MK_EINVAL, MK_ECUDA, MK_ESTATE, MK_EDEVICE = 0, -1, -2, -3, -4
DERR = {0: "none", 1: "wait_timeout", 2: "ring_timeout", 3: "token_range", 4: "aborted", 5: "bad_expert"}

# operator types and flags
OP_EMBED, OP_GEMV, OP_MLA_PREP, OP_MLA_ATTEND, OP_MLA_MERGE_UV, OP_ROUTER, OP_GATEUP, OP_W2_COMBINE, OP_STREAM, \
    OP_COPY, OP_MOE_UNITS, OP_MOE_COMBINE = range(1, 13)
F_NORM, F_RESIDUAL, F_ARGMAX, F_EXPERT, F_STATIC_IDS, F_EP, F_TC, F_FP8 = 1, 2, 4, 8, 16, 32, 64, 128

# ptr / ip indices (mirrors the enums of fleet_mk.h)
P = dict(
    emb=dict(W=0, TOKENS=1, OUT=2), emb_i=dict(V=0, H=1),
    gemv=dict(X=0, WNORM=1, W=2, RES=3, OUT=4, HOUT=5, TOKENS=6), gemv_i=dict(N=0, K=1),
    prep=dict(QKVA=0, WKVNORM=1, WUKT=2, COS=3, SIN=4, CKV=5, KPE=6, QLNOPE=7, QPE=8),
    prep_i=dict(NH=0, DN=1, DR=2, DC=3, SMAX=4),
    att=dict(QLNOPE=0, QPE=1, CKV=2, KPE=3, PARTIALS=4, SCORES=5),
    att_i=dict(NH=0, DC=1, DR=2, SMAX=3, SPLIT=4, HGROUP=5, NSPLITS=6, PROW=7, CPARTS=8),
    mrg=dict(PARTIALS=0, WUV=1, OUT=2), mrg_i=dict(NH=0, DV=1, DC=2, SPLIT=3, NSPLITS=4, PROW=5),
    rt=dict(X=0, WNORM=1, WGATE=2, HOUT=3, LOGITS=4, TOPKW=5, ROUTING=6, MASK=7, ROUTELOG=8, BIAS=9, LOGTAG=10,
            MASKTAG=11),
    rt_i=dict(H=0, E=1, TOPK=2, NFORCED=3, LAYER=4, LOGSTRIDE=5, LOGROWS=6),
    gu=dict(X=0, WNORM=1, W=2, MASK=3, MID=4, ACT=5, HOUT=6),
    gu_i=dict(K=0, I=1, GROUPS=2, ESTRIDE=3, NEXP=4, EPRANK=5, EPWORLD=6, SLOT0=7),
    w2=dict(ACT=0, W=1, MASK=2, TOPKW=3, XRES=4, OUT8=5, PEERS=6),
    w2_i=dict(H=0, I=1, SLOTS=2, ESTRIDE=3, NEXP=4, TOPK=5, EPRANK=6, EPWORLD=7, LAYER=8),
    st=dict(W=0, OUT=1), st_i=dict(ROWS=0, K=1),
    cp=dict(SRC=0, DST=1), cp_i=dict(N=0),
    mu=dict(X=0, WNORM=1, W13=2, W2F=3, MASK=4, SUMS=5, ACT=6, HOUT=7, MASKTAG=8, SCALE13=9),
    mu_i=dict(H=0, I=1, SLOT0=2, NSLOTS=3, NS=4, NEXP=5, EXP0=6, FIXED0=7, FTASKS=8),
    mc=dict(SUMS=0, TOPKW=1, XRES=2, OUT8=3, MASK=4, SCALE2=5), mc_i=dict(H=0, I=1, NS=2),
)


class MkOp(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("flags", ctypes.c_int32), ("ntasks", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("ptr", ctypes.c_void_p * 16), ("ip", ctypes.c_int64 * 16),
                ("fp", ctypes.c_double * 4)]


class MkConfig(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("num_ctas", ctypes.c_int32), ("wait_timeout_ns", ctypes.c_int64),
                ("trace", ctypes.c_int32), ("reserved", ctypes.c_int32 * 7)]


EP_MAX_RANKS, EP_MAX_TASKS = 8, 256


class MkEpPeers(ctypes.Structure):
    _fields_ = [("xch", ctypes.c_void_p * EP_MAX_RANKS), ("nranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("n_slots", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 3)]


class MkStatus(ctypes.Structure):
    _fields_ = [("error", ctypes.c_uint32), ("err_op", ctypes.c_uint32), ("err_task", ctypes.c_uint32),
                ("err_cta", ctypes.c_uint32), ("err_info", ctypes.c_uint32), ("aborted_ctas", ctypes.c_uint32),
                ("launches", ctypes.c_uint64), ("generation", ctypes.c_uint64)]

    def as_dict(self):
        d = {k: getattr(self, k) for k, _ in self._fields_}
        d["error_name"] = DERR.get(self.error, str(self.error))
        return d


class MkTraceRecord(ctypes.Structure):
    _fields_ = [("op", ctypes.c_uint32), ("task", ctypes.c_uint32), ("cta", ctypes.c_uint32),
                ("iter", ctypes.c_uint32), ("t_ready", ctypes.c_uint64), ("t_end", ctypes.c_uint64),
                ("t_body", ctypes.c_uint64), ("t_stages", ctypes.c_uint64), ("wait_ns", ctypes.c_uint64)]


EXPORTS = ["mk_version", "mk_last_error", "mk_create", "mk_add_op", "mk_finalize", "mk_launch", "mk_decode_token",
           "mk_status",
           "mk_reset", "mk_trace", "mk_op_tasks", "mk_destroy", "mk_debug_block_op", "mk_selftest_math",
           "mk_mla_decode_noalloc", "mk_set_op_deps", "mk_ep_alloc", "mk_ep_free", "mk_ep_ipc_handle",
           "mk_ep_ipc_open", "mk_ep_ipc_close"]

_lib = None


class MkError(RuntimeError):
    def __init__(self, code, msg, status=None):
        super().__init__(f"fleet_mk error {code}: {msg}")
        self.code = code
        self.status = status


def lib():
    """The loaded library (raises if it was not built: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `make -C {PKG / 'csrc'}` "
                                    "(or __graft_entry__.build())")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.mk_version.restype = ctypes.c_int
        L.mk_last_error.restype = ctypes.c_char_p
        L.mk_create.argtypes = [ctypes.POINTER(MkConfig), ctypes.POINTER(vp)]
        L.mk_add_op.argtypes = [vp, ctypes.POINTER(MkOp), ctypes.POINTER(i32)]
        L.mk_finalize.argtypes = [vp]
        L.mk_launch.argtypes = [vp, vp, i32, i32, vp]
        L.mk_decode_token.argtypes = [vp, vp, vp, i32, vp, vp, vp]
        L.mk_status.argtypes = [vp, ctypes.POINTER(MkStatus)]
        L.mk_reset.argtypes = [vp]
        L.mk_trace.argtypes = [vp, ctypes.POINTER(MkTraceRecord), i64, ctypes.POINTER(i64)]
        L.mk_op_tasks.argtypes = [vp, i32, ctypes.POINTER(i32)]
        L.mk_set_op_deps.argtypes = [vp, i32, ctypes.POINTER(i32), i32]
        L.mk_ep_alloc.argtypes = [i32, ctypes.c_size_t, ctypes.POINTER(vp)]
        L.mk_ep_free.argtypes = [vp]
        L.mk_ep_ipc_handle.argtypes = [vp, vp]
        L.mk_ep_ipc_open.argtypes = [i32, vp, ctypes.POINTER(vp)]
        L.mk_ep_ipc_close.argtypes = [vp]
        L.mk_destroy.argtypes = [vp]
        L.mk_debug_block_op.argtypes = [vp, i32]
        L.mk_selftest_math.argtypes = [i32, vp, vp, i64, vp]
        L.mk_mla_decode_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32,
                                            ctypes.c_float, vp]
        for name in EXPORTS:
            getattr(L, name).restype = ctypes.c_int if name != "mk_last_error" else ctypes.c_char_p
        _lib = L
    return _lib


def _check(rc, what):
    if rc != MK_OK:
        raise MkError(rc, f"{what}: {lib().mk_last_error().decode()}")


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def make_op(type_, flags=0, ptrs=None, ips=None, fps=None, ntasks=0):
    """An MkOp from {index: tensor-or-pointer}, {index: int}, {index: float}."""
    op = MkOp()
    op.type = type_
    op.flags = flags
    op.ntasks = ntasks
    for i, t in (ptrs or {}).items():
        op.ptr[i] = _ptr(t)
    for i, v in (ips or {}).items():
        op.ip[i] = int(v)
    for i, v in (fps or {}).items():
        op.fp[i] = float(v)
    return op


class MegaKernel:
    """One handle of the persistent decode kernel: operators, schedule, launches."""

    def __init__(self, device=0, num_ctas=0, wait_timeout_s=2.0, trace=False):
        cfg = MkConfig()
        cfg.device = int(device)
        cfg.num_ctas = int(num_ctas)
        cfg.wait_timeout_ns = int(wait_timeout_s * 1e9)
        cfg.trace = 1 if trace else 0
        h = ctypes.c_void_p()
        _check(lib().mk_create(ctypes.byref(cfg), ctypes.byref(h)), "mk_create")
        self.h = h
        self.device = device
        self.ops = []
        self.finalized = False
        self._keep = []            # tensors whose pointers the library holds

    def add(self, op, keep=()):
        idx = ctypes.c_int32()
        _check(lib().mk_add_op(self.h, ctypes.byref(op), ctypes.byref(idx)), f"mk_add_op #{len(self.ops)}")
        self.ops.append(op)
        self._keep.extend(keep)
        return idx.value

    def set_deps(self, op_index, deps):
        """Operator op_index waits for the earlier operators `deps` (1 or 2) instead of the previous one."""
        arr = (ctypes.c_int32 * len(deps))(*deps)
        _check(lib().mk_set_op_deps(self.h, op_index, arr, len(deps)), "mk_set_op_deps")

    def tasks(self, op_index):
        n = ctypes.c_int32()
        _check(lib().mk_op_tasks(self.h, op_index, ctypes.byref(n)), "mk_op_tasks")
        return n.value

    def finalize(self):
        _check(lib().mk_finalize(self.h), "mk_finalize")
        self.finalized = True

    def launch(self, iters=1, step=0, stream=None, meta_step=None):
        s = stream.cuda_stream if stream is not None and hasattr(stream, "cuda_stream") else (stream or 0)
        _check(lib().mk_launch(self.h, s, int(iters), int(step), _ptr(meta_step)), "mk_launch")

    def decode_token(self, tokens, step, token_in, token_out, stream=None, meta_step=None):
        """One token host to host (mk_decode_token): token_in / token_out are pinned int64 host
        tensors, tokens the device row the embedding reads."""
        s = stream.cuda_stream if stream is not None and hasattr(stream, "cuda_stream") else (stream or 0)
        _check(lib().mk_decode_token(self.h, s, _ptr(tokens), int(step), _ptr(token_in), _ptr(token_out),
                                     _ptr(meta_step)), "mk_decode_token")

    def status(self, raise_on_error=True):
        st = MkStatus()
        rc = lib().mk_status(self.h, ctypes.byref(st))
        if rc == MK_EDEVICE and not raise_on_error:
            return st.as_dict()
        if rc != MK_OK:
            raise MkError(rc, f"mk_status: {lib().mk_last_error().decode()}", st.as_dict())
        return st.as_dict()

    def reset(self):
        _check(lib().mk_reset(self.h), "mk_reset")

    def block_op(self, op_index):
        _check(lib().mk_debug_block_op(self.h, int(op_index)), "mk_debug_block_op")

    def trace(self, cap=1 << 20):
        n = ctypes.c_int64()
        _check(lib().mk_trace(self.h, None, 0, ctypes.byref(n)), "mk_trace")
        m = min(n.value, cap)
        buf = (MkTraceRecord * max(1, m))()
        _check(lib().mk_trace(self.h, buf, m, ctypes.byref(n)), "mk_trace")
        return [(r.op, r.task, r.cta, r.iter, r.t_ready, r.t_end, r.t_body, r.t_stages, r.wait_ns) for r in buf[:m]]

    def close(self):
        if getattr(self, "h", None):
            lib().mk_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ep_alloc(device, nbytes):
    p = ctypes.c_void_p()
    _check(lib().mk_ep_alloc(int(device), int(nbytes), ctypes.byref(p)), "mk_ep_alloc")
    return p.value


def ep_free(ptr):
    _check(lib().mk_ep_free(ctypes.c_void_p(ptr)), "mk_ep_free")


def ep_ipc_handle(ptr):
    buf = (ctypes.c_uint8 * 64)()
    _check(lib().mk_ep_ipc_handle(ctypes.c_void_p(ptr), buf), "mk_ep_ipc_handle")
    return bytes(buf)


def ep_ipc_open(device, handle):
    buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    p = ctypes.c_void_p()
    _check(lib().mk_ep_ipc_open(int(device), buf, ctypes.byref(p)), "mk_ep_ipc_open")
    return p.value


def ep_ipc_close(ptr):
    _check(lib().mk_ep_ipc_close(ctypes.c_void_p(ptr)), "mk_ep_ipc_close")


def selftest_math(fn, x, out, stream=None):
    """Run one of the device's deterministic-arithmetic routines over n values (device tensors)."""
    s = stream.cuda_stream if stream is not None and hasattr(stream, "cuda_stream") else 0
    _check(lib().mk_selftest_math(int(fn), _ptr(x), _ptr(out), int(x.numel()), s), "mk_selftest_math")


def mla_decode_noalloc(ql_nope, q_pe, c_kv, k_pe, w_uv, attn_out, pos, split, softmax_scale, stream=None):
    """MLA decode attention (split-KV partials, merge, W_uv) for callers that must not allocate
    device memory here: the partials live in the library's static device array (2 MiB), so nothing
    is allocated and calls that overlap on the GPU race. Same result as the MLA_ATTEND +
    MLA_MERGE_UV operators of the persistent kernel, bit for bit. Tensors are BF16 on the device."""
    nh, d_c = ql_nope.shape
    d_r = q_pe.shape[1]
    d_v = w_uv.shape[1]
    s = stream.cuda_stream if stream is not None and hasattr(stream, "cuda_stream") else (stream or 0)
    _check(lib().mk_mla_decode_noalloc(_ptr(ql_nope), _ptr(q_pe), _ptr(c_kv), _ptr(k_pe), _ptr(w_uv),
                                       _ptr(attn_out), nh, d_c, d_r, d_v, int(pos), int(split),
                                       float(softmax_scale), s), "mk_mla_decode_noalloc")
