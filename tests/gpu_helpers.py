"""Helpers of the GPU parity tests: seeded BF16 tensors, device <-> oracle conversion, and the
oracle fed from device-resident packed weights."""
import numpy as np
import torch

from oracle.detmath import from_bf16_bits


def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def rnd_bf16(gen, *shape, std=1.0, device="cuda:0"):
    return (torch.randn(*shape, generator=gen, device=device) * std).to(torch.bfloat16)


def np32(t):
    """A BF16/FP32 torch tensor as float32 numpy (BF16 values exactly)."""
    return t.detach().float().cpu().numpy()


def bits(t):
    """BF16 tensor -> uint16 patterns (numpy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def np_bits(a):
    """float32 numpy of BF16 values -> uint16 patterns."""
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def assert_bits_equal(got_t, want_np, what=""):
    g = bits(got_t).reshape(-1)
    w = np_bits(want_np).reshape(-1)
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, (f"{what}: {bad.size} of {g.size} BF16 values differ; first at {bad[:5]}: "
                           f"got {from_bf16_bits(g[bad[:5]])} want {from_bf16_bits(w[bad[:5]])}")


class DeviceWeights:
    """The oracle's weight accessors over device tensors (copied to the host on first use)."""

    def __init__(self, packed):
        self.packed = packed
        self.cache = {}

    def get(self, name):
        if name not in self.cache:
            self.cache[name] = np32(self.packed[name])
        return self.cache[name]

    def get_expert(self, name, e):
        key = (name, e)
        if key not in self.cache:
            self.cache[key] = np32(self.packed[name][e])
        return self.cache[key]


class DeviceFP8:
    """The oracle's FP8 expert accessor, fp8(l, e): each layer's W13 / W2 quantised on the device as
    the FP8 graph quantises them (pack_weights.quantize_e4m3), one expert's codes and scales copied
    to the host on use."""

    def __init__(self, packed):
        self.packed = packed
        self.layers = {}

    def __call__(self, l, e):
        from fleet.pack_weights import quantize_e4m3
        if l not in self.layers:
            self.layers[l] = quantize_e4m3(self.packed[f"W13_{l}"], 2) + quantize_e4m3(self.packed[f"W2_{l}"], 1)
        W13q, s13, W2q, s2 = self.layers[l]
        return (W13q[e].cpu().numpy(), s13[e].cpu().numpy(), W2q[e].cpu().numpy(),
                np.float32(s2[e, 0].item()))


def u16(t):
    """A BF16 device tensor as its uint16 bit patterns on the host."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class DeviceWeightBits:
    """The oracle's weight accessors over device tensors, as BF16 bit patterns (uint16 numpy, which
    the oracle's row dots read directly). Tensors other than the experts are copied once; a routed
    expert is copied on every use and only the always-selected (shared) experts are kept, so the host
    holds a few GB while the oracle decodes the 31 GB model."""

    def __init__(self, packed, keep_experts=()):
        self.packed = packed
        self.keep = set(keep_experts)
        self.cache = {}

    def get(self, name):
        if name not in self.cache:
            self.cache[name] = u16(self.packed[name])
        return self.cache[name]

    def get_expert(self, name, e):
        if e not in self.keep:
            return u16(self.packed[name][e])
        key = (name, e)
        if key not in self.cache:
            self.cache[key] = u16(self.packed[name][e])
        return self.cache[key]
