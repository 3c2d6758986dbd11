"""turbo_b200_attention_noalloc: the tensor-core attention for callers that
cannot allocate device memory (their framework's memory pool owns it, or
their serving loop may not allocate). The caller passes its own device
buffers; the kernel's scratch lives in the library's fixed device array.

Checked through the C ABI against the existing entry point
(turbo_b200_attention_check, which allocates its own buffers) on the same
data, two calls in a row, within the tests' tolerance for the same kernel,
and against attention computed in F64 on the host within the kernel tests'
bound. This file is collected last."""
import ctypes as C

import numpy as np
import pytest

from test_gpu_kernels import ref_attention
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

F16, BF16 = abi.TURBO_DTYPE_F16, abi.TURBO_DTYPE_BF16


def _entry():
    lib = runtime.library()
    f = lib.turbo_b200_attention_noalloc
    f.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                  C.c_int32, C.c_void_p, C.POINTER(C.c_int32), C.POINTER(abi.turbo_error)]
    f.restype = C.c_int32
    return f


def _case(seed, lens, heads, dtype):
    rng = np.random.default_rng(seed)
    T = int(sum(lens))
    qkv = rng.standard_normal((T, 3 * heads * 64)).astype(np.float32) * 2
    qkv = qkv.astype(np.float16).astype(np.float32) if dtype == F16 else models.from_bf16_bits(
        models.to_bf16_bits(qkv))
    live = (rng.random(T) > 0.1).astype(np.uint8)
    return qkv, live


def _noalloc(dtype, lens, qkv, live, heads, window):
    import torch
    dev = torch.device("cuda:0")
    tdt = torch.float16 if dtype == F16 else torch.bfloat16
    q = torch.from_numpy(qkv).to(dev, tdt).contiguous()
    ctx = torch.zeros((qkv.shape[0], heads * 64), dtype=tdt, device=dev)
    lv = torch.from_numpy(live).to(dev)
    ln = np.ascontiguousarray(lens, np.int32)
    fault = C.c_int32(-1)
    err = abi.new_error()
    torch.cuda.synchronize()
    rc = _entry()(dtype, q.data_ptr(), ctx.data_ptr(), lv.data_ptr(), ln.ctypes.data_as(C.c_void_p), len(ln), heads,
                  64, window, None, C.byref(fault), C.byref(err))
    assert rc == 0, err.message
    torch.cuda.synchronize()
    assert fault.value == 0
    return ctx.float().cpu().numpy()


@pytest.mark.parametrize("dtype", [F16, BF16])
def test_noalloc_attention_matches_the_allocating_entry_point_twice(dtype):
    import torch
    torch.cuda.init()
    for seed, lens, heads, window in [(1, [300, 5, 129, 512], 12, -1), (2, [77, 260], 4, 64)]:
        qkv, live = _case(seed, lens, heads, dtype)
        got = _noalloc(dtype, lens, qkv, live, heads, window)
        want = runtime.attention_check(dtype, 2, lens, qkv, live, heads, 64, window)
        scale = max(np.abs(want).max(), 1e-30)
        assert np.abs(got - want).max() / scale < (1.2e-2 if dtype == BF16 else 2e-3)
        exact = ref_attention(qkv, lens, live, heads, 64, window)
        scale = max(np.abs(exact).max(), 1e-30)
        assert np.abs(got - exact).max() / scale < (1.2e-2 if dtype == BF16 else 2e-3)


def test_noalloc_attention_refuses_unaligned_buffers_before_any_launch():
    import torch
    torch.cuda.init()
    qkv, live = _case(4, [64], 1, F16)
    q = torch.from_numpy(qkv).to("cuda:0", torch.float16)
    ctx = torch.zeros((64 * 64 + 8,), dtype=torch.float16, device="cuda:0")
    lv = torch.from_numpy(live).to("cuda:0")
    lens = np.full(1, 64, np.int32)
    for qp, cp, what in [(q.data_ptr() + 2, ctx.data_ptr(), b"qkv"), (q.data_ptr(), ctx.data_ptr() + 2, b"ctx")]:
        err = abi.new_error()
        rc = _entry()(F16, qp, cp, lv.data_ptr(), lens.ctypes.data_as(C.c_void_p), 1, 1, 64, -1, None, None,
                      C.byref(err))
        assert rc == abi.TURBO_E_INVALID_ARGUMENT and what in err.message
    assert not ctx.any().item()  # nothing was launched: ctx is untouched


def test_noalloc_attention_refuses_work_beyond_its_scratch():
    import torch
    torch.cuda.init()
    qkv, live = _case(3, [64], 1, F16)
    q = torch.from_numpy(qkv).to("cuda:0", torch.float16)
    ctx = torch.zeros((64, 64), dtype=torch.float16, device="cuda:0")
    lv = torch.from_numpy(live).to("cuda:0")
    # More 128-query tiles than the array holds: refused before any launch.
    lens = np.full(1, 128 * (65536 + 1), np.int32)
    err = abi.new_error()
    rc = _entry()(F16, q.data_ptr(), ctx.data_ptr(), lv.data_ptr(), lens.ctypes.data_as(C.c_void_p), 1, 1, 64, -1,
                  None, None, C.byref(err))
    assert rc == abi.TURBO_E_CAPACITY and b"scratch" in err.message
