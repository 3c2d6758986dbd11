"""The drop-in boundary: struct layouts equal the reference's, and the
library exports every symbol include/turbo_b200.h declares. CPU only: the
library is loaded but nothing is computed."""
import ctypes as C
import json
import re
import subprocess
from pathlib import Path

import pytest

from turboembed_b200 import abi, runtime

ROOT = Path(__file__).resolve().parents[1]
FIXTURE = json.loads((ROOT / "tests/golden/abi_offsets.json").read_text())


def test_ctypes_mirror_matches_the_reference_layout():
    for name, cls in abi.STRUCTS.items():
        want = FIXTURE[name]
        assert C.sizeof(cls) == want["__size__"], name
        for f, *_ in cls._fields_:
            assert getattr(cls, f).offset == want[f], (name, f)


def test_c_header_matches_the_reference_layout():
    import sys
    sys.path.insert(0, str(ROOT / "tests/golden"))
    from make_abi_fixture import probe
    got = probe(ROOT / "include", "turbo/turbo_abi.h")
    assert got == FIXTURE


@pytest.fixture(scope="module")
def lib():
    if not runtime.LIB_PATH.exists():
        from turboembed_b200 import build
        build.build()
    return runtime.library()


def declared_symbols():
    text = (ROOT / "include/turbo_b200.h").read_text()
    return set(re.findall(r"TB_EXPORT[^;(]*?\b(turbo_\w+)\s*[;(]", text))


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert {"turbo_cuda_backend", "turbo_cuda_allocations", "turbo_b200_gemm_check"} <= syms
    out = subprocess.run(["nm", "-D", "--defined-only", str(runtime.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines()}
    assert syms <= exported, syms - exported
    for s in syms:
        getattr(lib, s)


def test_table_is_complete_and_sized(lib):
    t = runtime.table()
    assert t.struct_size == C.sizeof(abi.turbo_backend) == FIXTURE["turbo_backend"]["__size__"]
    assert t.name == b"cuda"
    assert t.formats == 1  # TURBO_FORMAT_BIT(SAFETENSORS)
    # turbo_backend.h:38-44: each offered create has its release; ranges need session_open.
    for f in ["device_count", "device_info", "capability", "context_create", "context_release", "buffer_alloc",
              "buffer_import", "buffer_release", "buffer_export", "model_load", "model_release", "session_create",
              "session_release", "embed_write", "session_run", "buffer_read", "session_create_tuned",
              "session_open", "embed_write_ranges"]:
        assert C.cast(getattr(t, f), C.c_void_p).value, f


def test_device_count_without_a_gpu_is_zero_not_an_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert runtime.Backend().device_count() == 0


def test_capability_answers_without_a_device(lib):
    b = runtime.Backend()
    st, dt, opts, reason = b.capability(0, abi.TURBO_TASK_EMBED, abi.TURBO_PRECISION_FASTEST)
    # Fields 4, 5, 6, 9 and 10 honoured, as the reference's cuda cell (backend.cpp:400).
    assert st == abi.TURBO_CAP_EXPERIMENTAL and dt == abi.TURBO_DTYPE_F16 and opts == 0x338
    st, dt, opts, reason = b.capability(0, abi.TURBO_TASK_EXTRACTIVE_QA if hasattr(abi, "TURBO_TASK_EXTRACTIVE_QA") else 3,
                                        abi.TURBO_PRECISION_EXACT)
    assert st == abi.TURBO_CAP_UNSUPPORTED and reason


def test_table_offers_buffer_quantize(lib):
    # The device int8 / ubinary codes (turbo_backend.h:609-626) are offered:
    # the core quantizes device vectors through them instead of on the host.
    t = runtime.table()
    assert C.cast(t.buffer_quantize, C.c_void_p).value is not None
