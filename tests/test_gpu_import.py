"""buffer_import wraps caller memory without copying, under the reference
backend's rules (core/cuda/backend.cpp:630-692): a CUDA_PTR is memory of the
context's device imported as DEVICE (device or managed memory) or SHARED
(managed); a HOST_PTR is host memory, never DEVICE, page-locked when PINNED,
managed when SHARED. Every bad combination is refused on the host with
TURBO_E_INVALID_ARGUMENT (an unknown handle kind with TURBO_E_UNSUPPORTED)
before anything touches the memory; the good ones read back through
buffer_read."""
import numpy as np
import pytest

from turboembed_b200 import abi, runtime

pytestmark = pytest.mark.gpu

HOST, PINNED, DEVICE, SHARED = abi.TURBO_PLACE_HOST, abi.TURBO_PLACE_PINNED, abi.TURBO_PLACE_DEVICE, abi.TURBO_PLACE_SHARED
CUDA_PTR, HOST_PTR = abi.TURBO_HANDLE_CUDA_PTR, abi.TURBO_HANDLE_HOST_PTR
N = 4096


@pytest.fixture(scope="module")
def ctx():
    b = runtime.Backend()
    c = b.context(0)
    yield c
    c.release()


@pytest.fixture(scope="module")
def memory():
    import torch
    pattern = (np.arange(N) % 251).astype(np.uint8)
    dev = torch.from_numpy(pattern).to("cuda:0")
    pinned = torch.from_numpy(pattern).pin_memory()
    pageable = pattern.copy()
    torch.cuda.synchronize()
    return pattern, dev, pinned, pageable


def refused(ctx, placement, kind, address, code=abi.TURBO_E_INVALID_ARGUMENT, nbytes=N, aux=0, offset=0):
    with pytest.raises(runtime.TurboError) as e:
        ctx.import_buffer(placement, nbytes, kind, address, aux=aux, offset=offset)
    assert e.value.code == code, e.value
    return e.value.message


def test_null_handle_is_refused(ctx):
    assert "NULL" in refused(ctx, DEVICE, CUDA_PTR, 0)
    assert "NULL" in refused(ctx, HOST, HOST_PTR, 0)


def test_address_space_overflow_is_refused(ctx):
    assert "address space" in refused(ctx, DEVICE, CUDA_PTR, 2**64 - 64, offset=32)
    assert "address space" in refused(ctx, HOST, HOST_PTR, 2**64 - 4096, nbytes=8192)


def test_unknown_handle_kind_is_unsupported(ctx, memory):
    _, dev, _, _ = memory
    refused(ctx, DEVICE, 7, dev.data_ptr(), code=abi.TURBO_E_UNSUPPORTED)


def test_cuda_pointer_rules(ctx, memory):
    _, dev, pinned, pageable = memory
    d = dev.data_ptr()
    # aux names another device than the context's.
    assert "aux" in refused(ctx, DEVICE, CUDA_PTR, d, aux=1)
    # A CUDA_PTR is DEVICE or SHARED memory, never HOST or PINNED.
    assert "placement" in refused(ctx, HOST, CUDA_PTR, d)
    assert "placement" in refused(ctx, PINNED, CUDA_PTR, d)
    # SHARED needs managed memory; device memory is not.
    assert "managed" in refused(ctx, SHARED, CUDA_PTR, d)
    # Host memory named as a CUDA pointer.
    refused(ctx, DEVICE, CUDA_PTR, pageable.ctypes.data)
    refused(ctx, DEVICE, CUDA_PTR, pinned.data_ptr())


def test_host_pointer_rules(ctx, memory):
    _, dev, pinned, pageable = memory
    # A HOST_PTR is never DEVICE memory.
    assert "DEVICE" in refused(ctx, DEVICE, HOST_PTR, pinned.data_ptr())
    # PINNED needs page-locked memory.
    assert "page-locked" in refused(ctx, PINNED, HOST_PTR, pageable.ctypes.data)
    # SHARED needs managed memory.
    assert "managed" in refused(ctx, SHARED, HOST_PTR, pageable.ctypes.data)
    # Device memory named as host memory.
    assert "device memory" in refused(ctx, HOST, HOST_PTR, dev.data_ptr())


def test_good_imports_read_back(ctx, memory):
    pattern, dev, pinned, pageable = memory
    cases = [(DEVICE, CUDA_PTR, dev.data_ptr()), (PINNED, HOST_PTR, pinned.data_ptr()),
             (HOST, HOST_PTR, pageable.ctypes.data), (HOST, HOST_PTR, pinned.data_ptr())]
    for placement, kind, address in cases:
        b = ctx.import_buffer(placement, N, kind, address)
        assert np.array_equal(b.read(N), pattern), (placement, kind)
        # The handle exports back as what it wraps.
        if placement == DEVICE:
            h = b.export(CUDA_PTR)
            assert h.handle == address and h.aux == 0
        b.release()
    # An offset into device memory.
    b = ctx.import_buffer(DEVICE, 1024, CUDA_PTR, dev.data_ptr(), offset=512)
    assert np.array_equal(b.read(1024), pattern[512:1536])
    b.release()
    # Managed memory (the backend's own SHARED allocation) as SHARED and as DEVICE.
    own = ctx.buffer(SHARED, N)
    h = own.export(CUDA_PTR)
    for placement in (SHARED, DEVICE):
        b = ctx.import_buffer(placement, N, CUDA_PTR, h.handle, aux=h.aux)
        b.read(N)
        b.release()
    own.release()


def test_quantize_refuses_an_imported_host_buffer(ctx, memory):
    _, _, _, pageable = memory
    b = ctx.import_buffer(HOST, N, HOST_PTR, pageable.ctypes.data)
    with pytest.raises(runtime.TurboError) as e:
        b.quantize(abi.TURBO_QUANTIZE_UBINARY, 1, 64)
    assert e.value.code == abi.TURBO_E_INVALID_ARGUMENT
    b.release()


def test_memory_of_another_device_is_refused(ctx):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU: no memory of another device to name")
    other = torch.zeros(N, dtype=torch.uint8, device="cuda:1")
    torch.cuda.synchronize(1)
    assert "device 1" in refused(ctx, DEVICE, CUDA_PTR, other.data_ptr(), aux=0)
