"""Python handles over the `turbo_cuda_backend` table of libturbo_b200.so.

Every call goes through the C table exactly as the reference core calls a
backend (core/src/session/*.rs -> include/turbo/turbo_backend.h): this
module is a caller, not an implementation. It fails loudly when the
library is missing; there is no CPU fallback.
"""
import ctypes as C
from pathlib import Path

import numpy as np

from . import abi

LIB_PATH = Path(__file__).resolve().parent / "libturbo_b200.so"
_lib = None


class TurboError(RuntimeError):
    def __init__(self, code, field, message, what=""):
        super().__init__(f"{what}: {code} (field {field}): {message}")
        self.code, self.field, self.message = code, field, message


def library():
    """The loaded libturbo_b200.so (built in-tree by turboembed_b200/build.py)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `python -m turboembed_b200.build`")
        _lib = C.CDLL(str(LIB_PATH))
        _lib.turbo_cuda_allocations.restype = C.c_uint64
        _lib.turbo_cuda_fail_allocation.argtypes = [C.c_int32]
        _lib.turbo_cuda_arch_label.restype = C.c_char_p
        _lib.turbo_b200_gemm_check.argtypes = [
            C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
            C.c_void_p, C.c_void_p, C.c_uint32, C.POINTER(abi.turbo_error)]
        _lib.turbo_b200_attention_check.argtypes = [
            C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
            C.c_uint32, C.c_int32, C.c_void_p, C.POINTER(abi.turbo_error)]
    return _lib


def table():
    return abi.turbo_backend.in_dll(library(), "turbo_cuda_backend")


def _check(code, err, what):
    if code != abi.TURBO_OK:
        raise TurboError(code, err.field, err.message.decode(errors="replace"), what)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _i32p(a):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_int32))


class Backend:
    """The table, with each function raising TurboError on a failing status."""

    def __init__(self):
        self.t = table()

    def device_count(self):
        n, err = C.c_uint32(), abi.new_error()
        _check(self.t.device_count(C.byref(n), C.byref(err)), err, "device_count")
        return n.value

    def device_info(self, ordinal=0):
        info, err = abi.turbo_device_info(), abi.new_error()
        info.struct_size = C.sizeof(info)
        _check(self.t.device_info(ordinal, C.byref(info), C.byref(err)), err, "device_info")
        return info

    def capability(self, ordinal, task, precision):
        st, dt, opts, err = C.c_uint32(), C.c_uint32(), C.c_uint32(), abi.new_error()
        reason = C.create_string_buffer(160)
        _check(self.t.capability(ordinal, task, precision, C.byref(st), C.byref(dt), C.byref(opts), reason, 160,
                                 C.byref(err)), err, "capability")
        return st.value, dt.value, opts.value, reason.value.decode()

    def context(self, ordinal=0):
        return Context(self, ordinal)


class Context:
    def __init__(self, backend, ordinal=0):
        self.b, self.t = backend, backend.t
        self.h = C.c_void_p()
        self._log = abi.turbo_log_fn(lambda u, level, msg: None)
        err = abi.new_error()
        _check(self.t.context_create(ordinal, self._log, None, C.byref(self.h), C.byref(err)), err, "context_create")
        self.ordinal = ordinal

    def load(self, desc):
        """model_load of a ModelDesc (turboembed_b200.models)."""
        return Model(self, desc)

    def buffer(self, placement, nbytes):
        return Buffer(self, placement, nbytes)

    def import_buffer(self, placement, nbytes, kind, address, aux=0, offset=0):
        """buffer_import: wrap memory the caller owns (a CUDA_PTR of device
        `aux`, or a HOST_PTR) as a buffer of `placement`; nothing is copied."""
        d = abi.turbo_buffer_desc(C.sizeof(abi.turbo_buffer_desc), placement, abi.TURBO_DTYPE_U8, 1,
                                  (abi.u64 * 2)(nbytes, 0), nbytes)
        h = abi.turbo_native_handle(C.sizeof(abi.turbo_native_handle), kind, address, aux, offset)
        out, host, err = C.c_void_p(), C.c_void_p(), abi.new_error()
        _check(self.t.buffer_import(self.h, C.byref(d), C.byref(h), C.byref(out), C.byref(host), C.byref(err)), err,
               "buffer_import")
        b = Buffer(self, placement, nbytes, handle=out)
        b.host = host
        return b

    def release(self):
        if self.h:
            self.t.context_release(self.h)
            self.h = C.c_void_p()


class Buffer:
    def __init__(self, ctx, placement, nbytes, handle=None, host=None, owned=True):
        self.ctx, self.t = ctx, ctx.t
        self.placement, self.nbytes = placement, nbytes
        self.h, self.host = C.c_void_p(), C.c_void_p()
        self.owned = owned
        if handle is not None:
            self.h = handle
            return
        d = abi.turbo_buffer_desc(C.sizeof(abi.turbo_buffer_desc), placement, abi.TURBO_DTYPE_U8, 1,
                                  (abi.u64 * 2)(nbytes, 0), nbytes)
        err = abi.new_error()
        _check(self.t.buffer_alloc(ctx.h, C.byref(d), C.byref(self.h), C.byref(self.host), C.byref(err)), err,
               "buffer_alloc")

    def export(self, kind=abi.TURBO_HANDLE_CUDA_PTR):
        out, err = abi.turbo_native_handle(), abi.new_error()
        out.struct_size = C.sizeof(out)
        _check(self.t.buffer_export(self.h, kind, C.byref(out), C.byref(err)), err, "buffer_export")
        return out

    def read(self, nbytes, dst=None):
        dst = np.empty(nbytes, np.uint8) if dst is None else dst
        err = abi.new_error()
        _check(self.t.buffer_read(self.h, _ptr(dst), nbytes, C.byref(err)), err, "buffer_read")
        return dst

    def quantize(self, quantization, rows, dim, ranges=None, run=None):
        """buffer_quantize: int8 / ubinary codes of the first rows x dim F32
        values, into the buffer's leading bytes (core/src/quantize.rs)."""
        rg = None if ranges is None else np.ascontiguousarray(ranges, np.float32)
        err = abi.new_error()
        _check(self.t.buffer_quantize(self.h, quantization, None if rg is None else rg.ctypes.data_as(C.POINTER(C.c_float)),
                                      rows, dim, None if run is None else C.byref(run), C.byref(err)),
               err, "buffer_quantize")

    def release(self):
        if self.h and self.owned:
            self.t.buffer_release(self.h)
        self.h = C.c_void_p()


class Model:
    def __init__(self, ctx, desc):
        self.ctx, self.t, self.desc = ctx, ctx.t, desc
        self.h = C.c_void_p()
        err = abi.new_error()
        _check(self.t.model_load(ctx.h, C.byref(desc.struct), C.byref(self.h), C.byref(err)), err, "model_load")

    def session(self, max_batch, max_seq, precision, task=abi.TURBO_TASK_EMBED, max_ranges=0, cpu_threads=0,
                numerics=None):
        """session_open with turbo_backend_tuning.numerics_allowed = `numerics`,
        or the core's own table for the precision when None."""
        return Session(self, max_batch, max_seq, precision, task, max_ranges, cpu_threads, numerics)

    def release(self):
        if self.h:
            self.t.model_release(self.h)
            self.h = C.c_void_p()


# The numeric classes the core allows each precision (core/src/tuning.rs:23-36):
# what the core hands session_open in turbo_backend_tuning.numerics_allowed.
CORE_NUMERICS = {
    abi.TURBO_PRECISION_EXACT: abi.TURBO_NUMERIC_F32_FMA,
    abi.TURBO_PRECISION_MODEL: abi.TURBO_NUMERIC_F32_FMA,
    abi.TURBO_PRECISION_FASTEST: abi.TURBO_NUMERIC_F16_F32ACC | abi.TURBO_NUMERIC_F16_CHUNKACC,
}


class Session:
    """session_open, then embed_write / embed_write_ranges + session_run,
    reading the vectors back with buffer_read. `numerics_used` is what the
    backend reports its kernels compute in."""

    def __init__(self, model, max_batch, max_seq, precision, task, max_ranges, cpu_threads, numerics=None):
        self.model, self.t = model, model.t
        d = abi.turbo_backend_session_desc(C.sizeof(abi.turbo_backend_session_desc), task, max_batch, max_seq,
                                           precision, cpu_threads, max_ranges, 0)
        self.tuning = abi.turbo_backend_tuning()
        self.tuning.struct_size = C.sizeof(self.tuning)
        self.tuning.mode = abi.TURBO_AUTOTUNE_OFF
        self.tuning.numerics_allowed = CORE_NUMERICS[precision] if numerics is None else numerics
        cd, err = C.c_uint32(), abi.new_error()
        self.h = C.c_void_p()
        _check(self.t.session_open(model.h, C.byref(d), C.byref(self.tuning), C.byref(cd), C.byref(self.h),
                                   C.byref(err)), err, "session_open")
        self.compute_dtype = cd.value
        self.numerics_used = self.tuning.numerics_used
        self.choices = self.tuning.choices.decode(errors="replace")
        self.hidden = model.desc.hidden
        self._out_dim, self._count = 0, 0

    def _rows(self, ids, mask, types, pooling, normalize, output_dim, taps=0, tap_alone=0):
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        types = None if types is None else np.ascontiguousarray(types, np.int32)
        self._keep = (ids, mask, types)
        b, s = ids.shape
        r = abi.turbo_backend_embed_rows(C.sizeof(abi.turbo_backend_embed_rows), b, s, s, _i32p(ids), _i32p(mask),
                                         _i32p(types), pooling, normalize, output_dim or self.hidden, 0, taps, tap_alone)
        return r

    def write(self, ids, mask, types=None, pooling=abi.TURBO_POOLING_MEAN, normalize=abi.TURBO_NORMALIZE_L2,
              output_dim=0):
        r = self._rows(ids, mask, types, pooling, normalize, output_dim)
        err = abi.new_error()
        _check(self.t.embed_write(self.h, C.byref(r), C.byref(err)), err, "embed_write")
        self._out_dim, self._count = r.output_dim, r.batch

    def write_device(self, ids_ptr, mask_ptr, types_ptr, batch, seq, pooling=abi.TURBO_POOLING_MEAN,
                     normalize=abi.TURBO_NORMALIZE_L2, output_dim=0):
        """turbo_b200_embed_write_device: rows already in device memory
        ([batch, seq] i32 at the given device addresses; types may be 0)."""
        lib = library()
        f = lib.turbo_b200_embed_write_device
        f.argtypes = [C.c_void_p, C.POINTER(abi.turbo_backend_embed_rows), C.POINTER(abi.turbo_error)]
        i32 = C.POINTER(C.c_int32)
        r = abi.turbo_backend_embed_rows(C.sizeof(abi.turbo_backend_embed_rows), batch, seq, seq,
                                         C.cast(C.c_void_p(ids_ptr), i32), C.cast(C.c_void_p(mask_ptr), i32),
                                         C.cast(C.c_void_p(types_ptr), i32) if types_ptr else None, pooling,
                                         normalize, output_dim or self.hidden, 0, 0, 0)
        err = abi.new_error()
        _check(f(self.h, C.byref(r), C.byref(err)), err, "embed_write_device")
        self._out_dim, self._count = r.output_dim, r.batch

    def write_ranges(self, ids, mask, ranges, types=None, normalize=abi.TURBO_NORMALIZE_L2, output_dim=0, taps=0,
                     tap_alone=0):
        """embed_write_ranges; taps T > 1 pools each range from each of the
        last T layers ([T * ranges, output_dim] after the run), tap_alone 1
        from the model cut after layer L - T + 1 alone."""
        r = self._rows(ids, mask, types, abi.TURBO_POOLING_MEAN, normalize, output_dim, taps, tap_alone)
        rg = np.ascontiguousarray(ranges, np.uint32).reshape(-1, 3)
        self._keep_ranges = rg
        err = abi.new_error()
        _check(self.t.embed_write_ranges(self.h, C.byref(r), rg.ctypes.data_as(C.POINTER(abi.turbo_token_range)),
                                         len(rg), C.byref(err)), err, "embed_write_ranges")
        self._out_dim, self._count = r.output_dim, len(rg) * (taps if taps > 1 and not tap_alone else 1)

    def run(self):
        out, err = abi.turbo_backend_run(), abi.new_error()
        out.struct_size = C.sizeof(out)
        out.stage[abi.TURBO_EMBED_STAGE_TOKENIZE] = abi.TURBO_STAGE_UNUSED
        _check(self.t.session_run(self.h, C.byref(out), C.byref(err)), err, "session_run")
        self.last_run = out
        return out

    def read(self, out=None):
        """The last run's vectors, [count, output_dim] F32, via buffer_read."""
        n = self._count * self._out_dim
        if out is not None and (out.dtype != np.float32 or out.size != n or not out.flags.c_contiguous):
            raise ValueError(f"read into a contiguous F32 array of {n} values, not {out.dtype} x {out.size}")
        dst = np.empty(n, np.float32) if out is None else out
        err = abi.new_error()
        _check(self.t.buffer_read(self.last_run.output, _ptr(dst), n * 4, C.byref(err)), err, "buffer_read")
        return dst.reshape(self._count, self._out_dim)

    def set_head(self, cls_w, cls_b, pooler_w=None, pooler_b=None):
        """turbo_b200_session_set_head: the cross-encoder head on the device."""
        lib = library()
        f = lib.turbo_b200_session_set_head
        f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.POINTER(abi.turbo_error)]
        self._head = [None if a is None else np.ascontiguousarray(a, np.float32) for a in (pooler_w, pooler_b, cls_w)]
        err = abi.new_error()
        _check(f(self.h, _ptr(self._head[0]), _ptr(self._head[1]), _ptr(self._head[2]), float(np.asarray(cls_b).ravel()[0]),
                 C.byref(err)), err, "set_head")

    def head_scores(self, n=None):
        """The head's score of each of the last run's first n vectors."""
        lib = library()
        f = lib.turbo_b200_session_head_scores
        f.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.POINTER(abi.turbo_error)]
        n = self._count if n is None else n
        out = np.zeros(n, np.float32)
        err = abi.new_error()
        _check(f(self.h, n, _ptr(out), C.byref(err)), err, "head_scores")
        return out

    def embed(self, ids, mask, types=None, **kw):
        self.write(ids, mask, types, **kw)
        self.run()
        return self.read()

    def release(self):
        if self.h:
            self.t.session_release(self.h)
            self.h = C.c_void_p()


def gemm_check(dtype, variant, epi, a, w, bias=None, y_in=None, head_dim=0, pos=None, cos=None, sin=None):
    """turbo_b200_gemm_check: one GEMM on the device from host F32 operands."""
    lib = library()
    a = np.ascontiguousarray(a, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, K = a.shape
    N = w.shape[0]
    cols = N // 2 if epi == 3 else N
    y = np.zeros((M, cols), np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    y_in = None if y_in is None else np.ascontiguousarray(y_in, np.float32)
    pos = None if pos is None else np.ascontiguousarray(pos, np.int32)
    cos = None if cos is None else np.ascontiguousarray(cos, np.float32)
    sin = None if sin is None else np.ascontiguousarray(sin, np.float32)
    positions = 0 if cos is None else cos.shape[0]
    err = abi.new_error()
    rc = lib.turbo_b200_gemm_check(dtype, variant, epi, M, N, K, _ptr(a), _ptr(w), _ptr(bias), _ptr(y_in), _ptr(y),
                                   head_dim, _ptr(pos), _ptr(cos), _ptr(sin), positions, C.byref(err))
    _check(rc, err, "gemm_check")
    return y


def gemm_ln_check(dtype, a, w, bias, y_in, ln_w, ln_b, eps):
    """turbo_b200_gemm_ln_check: LN(y_in + a w^T + bias) * ln_w + ln_b on the
    fused tcgen05 GEMM (N = 768 or 1024)."""
    lib = library()
    f = lib.turbo_b200_gemm_ln_check
    f.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32] + [C.c_void_p] * 6 + [C.c_float, C.c_void_p,
                                                                                         C.POINTER(abi.turbo_error)]
    arrs = [np.ascontiguousarray(x, np.float32) for x in (a, w, bias, y_in, ln_w, ln_b)]
    M, K = arrs[0].shape
    N = arrs[1].shape[0]
    out = np.zeros((M, N), np.float32)
    err = abi.new_error()
    _check(f(dtype, M, N, K, *[_ptr(x) for x in arrs], eps, _ptr(out), C.byref(err)), err, "gemm_ln_check")
    return out


def gemm_ln_dual_check(dtype, a, w, bias, y_in, ln_w, ln_b, eps):
    """turbo_b200_gemm_ln_dual_check: (sum, LN(sum) * ln_w + ln_b) with
    sum = y_in + a w^T + bias, from the pre-norm fused GEMM (N = 768)."""
    lib = library()
    f = lib.turbo_b200_gemm_ln_dual_check
    f.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32] + [C.c_void_p] * 6 + [
        C.c_float, C.c_void_p, C.c_void_p, C.POINTER(abi.turbo_error)]
    arrs = [np.ascontiguousarray(x, np.float32) for x in (a, w, bias, y_in, ln_w, ln_b)]
    M, K = arrs[0].shape
    N = arrs[1].shape[0]
    total = np.zeros((M, N), np.float32)
    out = np.zeros((M, N), np.float32)
    err = abi.new_error()
    _check(f(dtype, M, N, K, *[_ptr(x) for x in arrs], eps, _ptr(total), _ptr(out), C.byref(err)), err,
           "gemm_ln_dual_check")
    return total, out


def attention_check(dtype, variant, lens, qkv, live, heads, head_dim, window=-1):
    lib = library()
    lens = np.ascontiguousarray(lens, np.int32)
    qkv = np.ascontiguousarray(qkv, np.float32)
    live = np.ascontiguousarray(live, np.uint8)
    T = int(lens.sum())
    ctx = np.zeros((T, heads * head_dim), np.float32)
    err = abi.new_error()
    rc = lib.turbo_b200_attention_check(dtype, variant, len(lens), _ptr(lens), _ptr(qkv), _ptr(live), heads,
                                        head_dim, window, _ptr(ctx), C.byref(err))
    _check(rc, err, "attention_check")
    return ctx
