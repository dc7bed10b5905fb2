"""Shared helpers of the parity tests."""
import numpy as np
import torch

# Attention tolerance against the fp32 recompute.
ATOL_MAX = 2e-2
ATOL_MEAN = 2e-3


def dev_bf16(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to("cuda", dtype)


def dev_i32(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.int32)).to("cuda")


def host(t):
    return t.float().cpu().numpy()


def assert_attn_close(got, want, what=""):
    err = np.abs(np.asarray(got, np.float32) - np.asarray(want, np.float32))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, \
        f"{what}: max|err| {err.max():.3e} mean {err.mean():.3e} first bad {np.unravel_index(err.argmax(), err.shape)}"
    return float(err.max()), float(err.mean())
