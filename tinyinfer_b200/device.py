"""ctypes binding of the device-layer C ABI (include/miniprefix_b200.h).

The library is loaded from this package directory; importing this module on a
machine without the built library fails loudly -- there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .synthetic import ModelConfig

HERE = os.path.dirname(os.path.abspath(__file__))
DEVICE_LIB = os.path.join(HERE, "libmpb200.so")

MP_OK, MP_ERR_INVALID, MP_ERR_CUDA, MP_ERR_NONFINITE, MP_ERR_BOUNDS, MP_ERR_TIMEOUT, MP_ERR_NOMEM, \
    MP_ERR_UNSUPPORTED = range(8)
ERROR_NAMES = {0: "MP_OK", 1: "MP_ERR_INVALID", 2: "MP_ERR_CUDA", 3: "MP_ERR_NONFINITE", 4: "MP_ERR_BOUNDS",
               5: "MP_ERR_TIMEOUT", 6: "MP_ERR_NOMEM", 7: "MP_ERR_UNSUPPORTED"}


class DeviceError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class ModelConfigC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "hidden", "intermediate", "heads", "kv_heads", "vocabulary",
                                         "context", "eos")] + [("rms_epsilon", C.c_float), ("rope_theta", C.c_float),
                                                               ("tied", C.c_int32)]


class RuntimeConfigC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("block_tokens", "max_blocks", "max_sequences", "table_stride",
                                         "max_step_tokens", "max_step_sequences")]


class SequenceDescC(C.Structure):
    _fields_ = [("slot", C.c_int32), ("start", C.c_int32), ("count", C.c_int32)]


class CountersC(C.Structure):
    _fields_ = [("forwards", C.c_uint64), ("forward_ms", C.c_double), ("kernel_launches", C.c_uint64),
                ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64), ("shared_prefix_rows", C.c_uint64),
                ("shared_prefix_tokens", C.c_uint64), ("host_prepare_ms", C.c_double), ("host_launch_ms", C.c_double),
                ("host_wait_ms", C.c_double)]


class TableEntryC(C.Structure):
    _fields_ = [("slot", C.c_int32), ("index", C.c_int32), ("block", C.c_int32)]


class TailCopyRegionC(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("destination", "source", "pitch", "width", "rows")]


_lib = None


def library() -> C.CDLL:
    """Load libmpb200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(DEVICE_LIB):
            raise ImportError(f"{DEVICE_LIB} is missing: run tinyinfer_b200.build.build() (no CPU fallback exists)")
        lib = C.CDLL(DEVICE_LIB)
        lib.mp_last_error.restype = C.c_char_p
        lib.mp_stream.restype = C.c_void_p
        lib.mp_stream.argtypes = [C.c_void_p]
        lib.mp_create.argtypes = [C.c_int, C.POINTER(ModelConfigC), C.POINTER(RuntimeConfigC), C.POINTER(C.c_void_p)]
        lib.mp_destroy.argtypes = [C.c_void_p]
        lib.mp_set_weight.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        lib.mp_finalize_weights.argtypes = [C.c_void_p]
        lib.mp_table_write.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int32]
        lib.mp_cow_copy.argtypes = [C.c_void_p, C.c_void_p, C.c_int32]
        lib.mp_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                                   C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32]
        lib.mp_forward_prepare.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32,
                                           C.c_void_p, C.c_int32]
        lib.mp_cow_timing.argtypes = [C.c_void_p, C.c_int32]
        lib.mp_read_counters.argtypes = [C.c_void_p, C.POINTER(CountersC), C.c_int32]
        lib.mp_cow_elapsed.argtypes = [C.c_void_p, C.POINTER(C.c_float)]
        lib.mp_forward_launch.argtypes = [C.c_void_p]
        lib.mp_forward_collect.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32]
        lib.mp_sync.argtypes = [C.c_void_p, C.c_int32]
        lib.mp_inject_wait_timeout.argtypes = [C.c_void_p, C.c_int32]
        lib.mp_kv_pools.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_uint64)]
        lib.mp_kv_read.argtypes = [C.c_void_p, C.c_int32, C.c_uint64, C.c_uint64, C.c_void_p]
        lib.mp_kv_write.argtypes = [C.c_void_p, C.c_int32, C.c_uint64, C.c_uint64, C.c_void_p]
        lib.mp_timer_mark.argtypes = [C.c_void_p]
        lib.mp_timer_elapsed.argtypes = [C.c_void_p, C.POINTER(C.c_float)]
        lib.mp_profile_enable.argtypes = [C.c_void_p, C.c_int32]
        lib.mp_set_shared_prefix.argtypes = [C.c_void_p, C.c_int32, C.c_int32]
        lib.mp_profile_read_gemm.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                             C.POINTER(C.c_float), C.POINTER(C.c_int32)]
        lib.mp_profile_read.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                        C.POINTER(C.c_double)]
        lib.mp_paged_attention_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                                  C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32,
                                                  C.c_void_p, C.c_int32, C.c_void_p]
        lib.mp_paged_attention_status.argtypes = [C.c_void_p]
        lib.mp_paged_attention_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32,
                                                   C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                                   C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
        lib.mp_gemm_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]
        _lib = lib
    return _lib


def last_error() -> str:
    return library().mp_last_error().decode()


def check(rc: int) -> None:
    if rc != MP_OK:
        raise DeviceError(rc, last_error())


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def model_config_c(c: ModelConfig) -> ModelConfigC:
    return ModelConfigC(c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.vocabulary, c.context, c.eos,
                        c.rms_epsilon, c.rope_theta, int(c.tied))


class DeviceContext:
    """One mp_context: weights, K/V pools, block tables and the step workspace on one GPU."""

    def __init__(self, config: ModelConfig, *, device: int = 0, block_tokens: int = 16, max_blocks: int = 128,
                 max_sequences: int = 64, max_step_tokens: int = 512, max_step_sequences: int = 64,
                 table_stride: int | None = None):
        self.lib = library()
        self.config = config
        if table_stride is None:
            table_stride = -(-config.context // block_tokens)
        self.runtime = RuntimeConfigC(block_tokens, max_blocks, max_sequences, table_stride, max_step_tokens,
                                      max_step_sequences)
        h = C.c_void_p()
        check(self.lib.mp_create(device, C.byref(model_config_c(config)), C.byref(self.runtime), C.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            self.lib.mp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_weights(self, weights: dict) -> None:
        for name, arr in weights.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            check(self.lib.mp_set_weight(self.h, name.encode(), _ptr(a), a.size))
        check(self.lib.mp_finalize_weights(self.h))

    def table_write(self, slot: int, first: int, blocks) -> None:
        b = np.ascontiguousarray(blocks, dtype=np.int32)
        check(self.lib.mp_table_write(self.h, slot, first, _ptr(b), len(b)))

    def cow_copy(self, regions) -> None:
        arr = (TailCopyRegionC * len(regions))(*[TailCopyRegionC(*r) for r in regions])
        check(self.lib.mp_cow_copy(self.h, arr, len(regions)))

    @staticmethod
    def _extras(entries, regions):
        e = (TableEntryC * max(1, len(entries)))(*[TableEntryC(*x) for x in entries])
        r = (TailCopyRegionC * max(1, len(regions)))(*[TailCopyRegionC(*x) for x in regions])
        return e, len(entries), r, len(regions)

    def forward(self, sequences, tokens, *, entries=(), regions=(), logits: bool = True, timeout_ms: int = 60000):
        """sequences: list of (slot, start, count); entries: (slot, index, block) table
        writes; regions: COW regions. Returns (tokens, finite, logits|None, rc)."""
        n = len(sequences)
        descs = (SequenceDescC * n)(*[SequenceDescC(*s) for s in sequences])
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out_t = np.zeros(n, dtype=np.int32)
        out_f = np.zeros(n, dtype=np.int32)
        out_l = np.zeros((n, self.config.vocabulary), dtype=np.float32) if logits else None
        e, ne, r, nr = self._extras(entries, regions)
        rc = self.lib.mp_forward(self.h, descs, n, _ptr(toks), e, ne, r, nr, _ptr(out_t), _ptr(out_f),
                                 _ptr(out_l) if logits else None, timeout_ms)
        if rc not in (MP_OK, MP_ERR_NONFINITE):
            check(rc)
        return out_t, out_f.astype(bool), out_l, rc

    def prepare(self, sequences, tokens, entries=(), regions=()) -> None:
        n = len(sequences)
        descs = (SequenceDescC * n)(*[SequenceDescC(*s) for s in sequences])
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        e, ne, r, nr = self._extras(entries, regions)
        check(self.lib.mp_forward_prepare(self.h, descs, n, _ptr(toks), e, ne, r, nr))

    def launch(self) -> None:
        check(self.lib.mp_forward_launch(self.h))

    def collect(self, n: int, logits: bool = False, timeout_ms: int = 60000):
        out_t = np.zeros(n, dtype=np.int32)
        out_f = np.zeros(n, dtype=np.int32)
        out_l = np.zeros((n, self.config.vocabulary), dtype=np.float32) if logits else None
        rc = self.lib.mp_forward_collect(self.h, _ptr(out_t), _ptr(out_f), _ptr(out_l) if logits else None,
                                         timeout_ms)
        if rc not in (MP_OK, MP_ERR_NONFINITE):
            check(rc)
        return out_t, out_f.astype(bool), out_l, rc

    def sync(self, timeout_ms: int = 60000) -> None:
        check(self.lib.mp_sync(self.h, timeout_ms))

    def inject_wait_timeout(self, wait_us: int) -> None:
        """Failure-path tests: the next forward's first GEMM issues no copies and its
        bounded waits run out after wait_us microseconds (mp_inject_wait_timeout)."""
        check(self.lib.mp_inject_wait_timeout(self.h, wait_us))

    def pools(self):
        k, v, n = C.c_void_p(), C.c_void_p(), C.c_uint64()
        check(self.lib.mp_kv_pools(self.h, C.byref(k), C.byref(v), C.byref(n)))
        return k.value, v.value, n.value

    def kv_read(self, pool: int, offset: int, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        check(self.lib.mp_kv_read(self.h, pool, offset, count, _ptr(out)))
        return out

    def kv_write(self, pool: int, offset: int, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        check(self.lib.mp_kv_write(self.h, pool, offset, a.size, _ptr(a)))

    def stream(self) -> int:
        return self.lib.mp_stream(self.h)

    def timer_mark(self) -> None:
        check(self.lib.mp_timer_mark(self.h))

    def timer_elapsed(self) -> float:
        ms = C.c_float()
        check(self.lib.mp_timer_elapsed(self.h, C.byref(ms)))
        return ms.value

    def profile(self, enabled: bool) -> None:
        check(self.lib.mp_profile_enable(self.h, int(enabled)))

    def profile_read(self):
        ms, n, b = C.c_float(), C.c_int32(), C.c_double()
        check(self.lib.mp_profile_read(self.h, C.byref(ms), C.byref(n), C.byref(b)))
        return ms.value, n.value, b.value

    def shared_prefix(self, min_rows: int, min_tokens: int = 128) -> None:
        """Shared-prefix attention for groups of >= min_rows rows (0: off, the default)."""
        check(self.lib.mp_set_shared_prefix(self.h, min_rows, min_tokens))


class ContextView:
    """Timing and counters of a device context owned elsewhere (e.g. by an engine)."""

    def __init__(self, handle):
        self.lib = library()
        self.h = C.c_void_p(handle)

    def timer_mark(self) -> None:
        check(self.lib.mp_timer_mark(self.h))

    def timer_elapsed(self) -> float:
        ms = C.c_float()
        check(self.lib.mp_timer_elapsed(self.h, C.byref(ms)))
        return ms.value

    def profile(self, enabled: bool) -> None:
        check(self.lib.mp_profile_enable(self.h, int(enabled)))

    def profile_read(self):
        ms, n, b = C.c_float(), C.c_int32(), C.c_double()
        check(self.lib.mp_profile_read(self.h, C.byref(ms), C.byref(n), C.byref(b)))
        return ms.value, n.value, b.value

    def profile_read_gemm(self):
        """(layer GEMM ms, intervals, LM head ms, head launches) since the last read."""
        g, n, h, k = C.c_float(), C.c_int32(), C.c_float(), C.c_int32()
        check(self.lib.mp_profile_read_gemm(self.h, C.byref(g), C.byref(n), C.byref(h), C.byref(k)))
        return g.value, n.value, h.value, k.value

    def counters(self, reset: bool = False) -> dict:
        out = CountersC()
        check(self.lib.mp_read_counters(self.h, C.byref(out), int(reset)))
        return {k: getattr(out, k) for k, _ in CountersC._fields_}

    def shared_prefix(self, min_rows: int, min_tokens: int = 128) -> None:
        """Shared-prefix attention for groups of >= min_rows rows (0: off, the default)."""
        check(self.lib.mp_set_shared_prefix(self.h, min_rows, min_tokens))

    def sync(self, timeout_ms: int = 600000) -> None:
        check(self.lib.mp_sync(self.h, timeout_ms))


def paged_attention_decode(q_ptr: int, keys_ptr: int, values_ptr: int, layers: int, layer: int, block_tokens: int,
                           max_blocks: int, tables_ptr: int, table_stride: int, lengths, out_ptr: int,
                           pages_per_split: int = 0, stream: int | None = None) -> None:
    """The decode operator on caller device pointers (see mp_paged_attention_decode)."""
    lib = library()
    lens = np.ascontiguousarray(lengths, dtype=np.int32)
    check(lib.mp_paged_attention_decode(q_ptr, keys_ptr, values_ptr, layers, layer, block_tokens, max_blocks,
                                        tables_ptr, table_stride, _ptr(lens), len(lens), out_ptr, pages_per_split,
                                        stream))


def paged_attention_prefill(q_ptr: int, keys_ptr: int, values_ptr: int, layers: int, layer: int, block_tokens: int,
                            max_blocks: int, tables_ptr: int, table_stride: int, starts, counts, out_ptr: int,
                            stream: int | None = None) -> None:
    """The prefill operator on caller device pointers (see mp_paged_attention_prefill)."""
    lib = library()
    st = np.ascontiguousarray(starts, dtype=np.int32)
    ct = np.ascontiguousarray(counts, dtype=np.int32)
    check(lib.mp_paged_attention_prefill(q_ptr, keys_ptr, values_ptr, layers, layer, block_tokens, max_blocks,
                                         tables_ptr, table_stride, _ptr(st), _ptr(ct), len(st), out_ptr, stream))


def gemm_f32(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, stream: int | None = None) -> None:
    """C = A . B^T on device buffers through the 3xTF32 tensor-core GEMM (test/tool entry)."""
    check(library().mp_gemm_f32(a_ptr, b_ptr, c_ptr, m, n, k, stream))


def paged_attention_status(stream: int | None = None) -> int:
    return library().mp_paged_attention_status(stream)
