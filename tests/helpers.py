"""Shared helpers for the parity tests."""
import numpy as np


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# Tolerance for fp32-accumulated matvec / attention outputs against the
# reference CPU path (relative L2 <= 1e-3).
REL_L2_TOL = 1e-3


def to_dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def from_dev(t):
    return t.detach().cpu().numpy()


def device_x(x, group=32):
    """The x the Q4_K / Q6_K matvecs multiply: per sub-block of `group`
    columns, s = max|x| / 127 and x ~ s (x0 + x1 / 256 + x2 / 65536), the
    three int8 limbs of v = x / s taken by rounding to nearest (a middle limb
    of 128 carries into x0) -- a model of the device quantiser
    (guanaco_b200/csrc/gb_mt.cuh: limbs), used to check that the kernels
    compute W . x~ up to fp32 rounding."""
    x = np.asarray(x, np.float32).reshape(-1, group)
    mx = np.abs(x).max(axis=1, keepdims=True)
    with np.errstate(divide="ignore"):
        inv = np.where(mx > 0, np.float32(127) / mx, np.float32(0)).astype(np.float32)
    v = (x * inv).astype(np.float32)
    x0 = np.rint(v)
    t1 = ((v - x0) * np.float32(256)).astype(np.float32)
    x1 = np.rint(t1)
    x2 = np.clip(np.rint((t1 - x1) * np.float32(256)), -128, 127)
    s = (mx / np.float32(127)).astype(np.float32)
    return ((x0 + x1 / 256.0 + x2 / 65536.0) * s).astype(np.float32).ravel()


def read_device(ptr: int, count: int, dtype=np.float32) -> np.ndarray:
    """count elements at a raw device address (e.g. a model's KV cache) as a
    host array, through the CUDA runtime's cudaMemcpy."""
    from cuda.bindings import runtime as rt

    out = np.empty(count, dtype=dtype)
    (err,) = rt.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess, err
    return out
