"""ctypes binding of the host-layer C ABI (include/miniprefix_b200_host.h).

Python mirrors of the reference MiniPrefix classes, backed by the C++ host layer:
  PrefixCache  -- KvBlockPool + ExactPrefixCache over named sequences
  KVManager    -- KVManager with Append transactions (``call(op, ...)`` API)
  Runner       -- ModelRunner: ``Runner.b200(...)`` on a GPU, or ``Runner.scripted(...)``
  Engine       -- Engine (takes ownership of a Runner)
Errors raise :class:`HostError` carrying the C++ exception class as ``code``
(-1 invalid_argument, -2 logic_error, -3 KvCapacityError, -4 runtime_error,
-5 out_of_range, -6 other) and its message.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import device as _device
from .synthetic import ModelConfig

HERE = os.path.dirname(os.path.abspath(__file__))
HOST_LIB = os.path.join(HERE, "libmpb200_host.so")

RUNNER_STATS_FIELDS = (
    "live_sequences", "live_kv_bytes", "peak_kv_bytes", "forward_tokens", "device_weight_bytes",
    "weight_uploaded_bytes", "token_uploaded_bytes", "kv_uploaded_bytes", "logits_downloaded_bytes",
    "device_allocations", "device_workspace_bytes", "kv_block_tokens", "kv_total_blocks", "kv_live_blocks",
    "kv_peak_blocks", "kv_reserved_bytes", "block_table_uploaded_bytes", "block_table_device_bytes",
    "prefix_cache_capacity", "kv_cached_blocks", "kv_cache_only_blocks", "prefix_hits", "prefix_misses",
    "prefix_reused_tokens", "prefix_evictions")
KV_STATS_FIELDS = (
    "live_sequences", "live_kv_bytes", "peak_kv_bytes", "forward_tokens", "kv_block_tokens", "kv_total_blocks",
    "kv_live_blocks", "kv_peak_blocks", "kv_reserved_bytes", "prefix_cache_capacity", "kv_cached_blocks",
    "kv_cache_only_blocks", "prefix_hits", "prefix_misses", "prefix_reused_tokens", "prefix_evictions")
COST_FIELDS = ("lookup_calls", "lookup_ns", "publish_calls", "publish_ns", "cow_pages", "cow_bytes",
               "cow_copy_ns", "cow_timed_copies")
CACHE_STATS_FIELDS = ("size", "index_nodes", "key_token_bytes", "hits", "misses", "reused_tokens", "evictions",
                      "cache_only_blocks", "live_blocks", "peak_blocks", "free_blocks")
ADMISSION = ("Ready", "Wait", "Impossible")
FINISH = ("Eos", "Length", "Cancelled", "Error")


class HostError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


_lib = None


def library() -> C.CDLL:
    global _lib
    if _lib is None:
        _device.library()  # loads libmpb200.so first (dependency)
        if not os.path.exists(HOST_LIB):
            raise ImportError(f"{HOST_LIB} is missing: run tinyinfer_b200.build.build()")
        lib = C.CDLL(HOST_LIB)
        lib.mph_last_error.restype = C.c_char_p
        for name in ("mph_cache_new", "mph_kv_new", "mph_runner_new_b200", "mph_runner_new_scripted",
                     "mph_engine_new", "mph_runner_new_b200_file"):
            getattr(lib, name).restype = C.c_void_p
        lib.mph_runner_new_b200_file.argtypes = [C.c_int32, C.c_char_p] + [C.c_int32] * 7
        lib.mph_cache_new.argtypes = [C.c_int32] * 5
        lib.mph_kv_new.argtypes = [C.c_int32] * 7
        lib.mph_runner_new_b200.argtypes = [C.c_int32, C.POINTER(_device.ModelConfigC)] + [C.c_int32] * 7
        lib.mph_runner_new_scripted.argtypes = [C.c_int32] * 7
        lib.mph_engine_new.argtypes = [C.c_void_p] + [C.c_int32] * 4
        lib.mph_runner_set_weight.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        for name in ("mph_cache_reuse", "mph_kv_reuse_prefix", "mph_kv_offset", "mph_runner_reuse_prefix",
                     "mph_runner_regions", "mph_engine_poll", "mph_engine_poll_compact"):
            getattr(lib, name).restype = C.c_long
        for name in ("mph_kv_reserve", "mph_runner_reserve"):
            getattr(lib, name).argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        lib.mph_engine_device.restype = C.c_void_p
        lib.mph_engine_device.argtypes = [C.c_void_p]
        lib.mph_engine_submit.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int32, C.c_uint32, C.c_int32]
        _lib = lib
    return _lib


def _ids(x) -> bytes:
    return x.encode() if isinstance(x, str) else x


def _toks(tokens):
    a = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
    return a, a.ctypes.data_as(C.c_void_p), len(a)


def _vp(h):
    return C.c_void_p(h)


class _Base:
    def __init__(self):
        self.lib = library()

    def error(self) -> str:
        return self.lib.mph_last_error().decode()

    def check(self, rc):
        if rc < 0:
            raise HostError(int(rc), self.error())
        return rc


class PrefixCache(_Base):
    """KvBlockPool + ExactPrefixCache with named sequences."""

    def __init__(self, block_tokens, max_blocks, prefix_blocks, layers=1, width=1):
        super().__init__()
        h = self.lib.mph_cache_new(block_tokens, max_blocks, prefix_blocks, layers, width)
        if not h:
            raise HostError(-1, self.error())
        self.h = _vp(h)
        self.max_blocks = max_blocks

    def close(self):
        if self.h:
            self.lib.mph_cache_free(self.h)
            self.h = None

    def append(self, seq, tokens):
        a, p, n = _toks(tokens)
        self.check(self.lib.mph_cache_append(self.h, _ids(seq), p, n))

    def publish(self, seq):
        self.check(self.lib.mph_cache_publish(self.h, _ids(seq)))

    def reuse(self, seq, prompt):
        a, p, n = _toks(prompt)
        return self.check(self.lib.mph_cache_reuse(self.h, _ids(seq), p, n))

    def release(self, seq):
        self.check(self.lib.mph_cache_release(self.h, _ids(seq)))

    def evict_one(self):
        return bool(self.check(self.lib.mph_cache_evict_one(self.h)))

    def journal(self, op):
        """Undo window: 'begin', 'rollback' (to the state at begin) or 'end'."""
        self.check(self.lib.mph_cache_journal(self.h, {"begin": 0, "rollback": 1, "end": 2}[op]))

    def clear(self):
        self.lib.mph_cache_clear(self.h)

    def stats(self):
        out = (C.c_uint64 * 11)()
        self.lib.mph_cache_stats(self.h, out)
        return dict(zip(CACHE_STATS_FIELDS, list(out)))

    def references(self):
        out = (C.c_uint64 * self.max_blocks)()
        self.check(self.lib.mph_cache_references(self.h, out, self.max_blocks))
        return list(out)

    def define(self, seq, used, tokens, blocks):
        """Set a sequence verbatim (no page accounting) to build malformed inputs."""
        a, p, n = _toks(tokens)
        b, q, m = _toks(blocks)
        self.check(self.lib.mph_cache_define(self.h, _ids(seq), int(used), p, n, q, m))

    def sequence(self, seq):
        used = C.c_int32()
        blocks = (C.c_int32 * 65536)()
        toks = (C.c_int32 * 65536)()
        n = self.check(self.lib.mph_cache_sequence(self.h, _ids(seq), C.byref(used), blocks, 65536, toks, 65536))
        return used.value, list(blocks[:n]), list(toks[:used.value])


class KVManager(_Base):
    """KVManager; ``call(op, *args)`` returns (code, result) without raising."""

    def __init__(self, block_tokens, max_blocks, prefix_blocks, layers, width, context, vocabulary):
        super().__init__()
        h = self.lib.mph_kv_new(block_tokens, max_blocks, prefix_blocks, layers, width, context, vocabulary)
        if not h:
            raise HostError(-1, self.error())
        self.h = _vp(h)

    def close(self):
        if self.h:
            self.lib.mph_kv_free(self.h)
            self.h = None

    def call(self, op: str, *args):
        L = self.lib
        if op == "reserve":
            rc = L.mph_kv_reserve(self.h, _ids(args[0]), C.c_size_t(args[1]))
            return rc, (ADMISSION[rc] if rc >= 0 else None)
        if op == "release_reservation":
            return L.mph_kv_release_reservation(self.h, _ids(args[0])), None
        if op == "create":
            return L.mph_kv_create(self.h, _ids(args[0])), None
        if op == "fork":
            return L.mph_kv_fork(self.h, _ids(args[0]), _ids(args[1])), None
        if op == "reuse_prefix":
            a, p, n = _toks(args[1])
            rc = L.mph_kv_reuse_prefix(self.h, _ids(args[0]), p, n)
            return (rc, rc) if rc < 0 else (0, rc)
        if op == "cache_prefix":
            return L.mph_kv_cache_prefix(self.h, _ids(args[0])), None
        if op == "clear_prefix_cache":
            return L.mph_kv_clear_prefix_cache(self.h), None
        if op == "append":
            a, p, n = _toks(args[1])
            tail = (C.c_long * 3)()
            region = (C.c_size_t * 5)()
            rc = L.mph_kv_append(self.h, _ids(args[0]), p, n, int(args[2]), tail, region)
            return rc, (tuple(tail), tuple(region) if tail[0] >= 0 and args[2] != 2 else None)
        if op == "reset_sequence":
            return L.mph_kv_reset_sequence(self.h, _ids(args[0])), None
        if op == "release":
            return L.mph_kv_release(self.h, _ids(args[0])), None
        if op == "clear":
            return L.mph_kv_clear(self.h), None
        raise ValueError(op)

    def stats(self):
        out = (C.c_size_t * 16)()
        self.lib.mph_kv_stats(self.h, out)
        return dict(zip(KV_STATS_FIELDS, list(out)))

    def sequence(self, id):
        used = C.c_int32()
        blocks = (C.c_int32 * 65536)()
        rc = self.lib.mph_kv_sequence(self.h, _ids(id), C.byref(used), blocks, 65536)
        if rc < 0:
            return None
        return used.value, list(blocks[:rc])


class Runner(_Base):
    """A ModelRunner handle. ``b200()`` drives the GPU; ``scripted()`` is device-free."""

    def __init__(self, handle, vocabulary, kind):
        super().__init__()
        self.h = _vp(handle)
        self.vocabulary = vocabulary
        self.kind = kind
        self.owned = True

    @classmethod
    def b200(cls, config: ModelConfig, weights: dict | None, *, context: int, block_tokens=16, max_blocks=128,
             prefix_blocks=0, device=0, max_sequences=256, max_step_tokens=4096, max_step_sequences=256):
        lib = library()
        m = _device.model_config_c(config)
        h = lib.mph_runner_new_b200(device, C.byref(m), context, block_tokens, max_blocks, prefix_blocks,
                                    max_sequences, max_step_tokens, max_step_sequences)
        if not h:
            raise HostError(-1, lib.mph_last_error().decode())
        r = cls(h, config.vocabulary, "b200")
        if weights is not None:
            r.load_weights(weights)
        return r

    @classmethod
    def b200_from_file(cls, path: str, *, context: int, block_tokens=16, max_blocks=128, prefix_blocks=0, device=0,
                       max_sequences=256, max_step_tokens=4096, max_step_sequences=256):
        """A B200 runner built from an MPFX0001 model file (the reference's
        make_cuda_runner(ModelWeights::load(path), context, kv))."""
        from . import mpfx

        cfg = mpfx.read_config(path)
        lib = library()
        h = lib.mph_runner_new_b200_file(device, path.encode(), context, block_tokens, max_blocks, prefix_blocks,
                                         max_sequences, max_step_tokens, max_step_sequences)
        if not h:
            raise HostError(-1, lib.mph_last_error().decode())
        r = cls(h, cfg.vocabulary, "b200")
        r.config = cfg
        return r

    @classmethod
    def scripted(cls, vocabulary, context, layers, width, block_tokens=16, max_blocks=128, prefix_blocks=0):
        lib = library()
        h = lib.mph_runner_new_scripted(vocabulary, context, layers, width, block_tokens, max_blocks, prefix_blocks)
        if not h:
            raise HostError(-1, lib.mph_last_error().decode())
        return cls(h, vocabulary, "scripted")

    def load_weights(self, weights: dict):
        for name, arr in weights.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            self.check(self.lib.mph_runner_set_weight(self.h, name.encode(), a.ctypes.data_as(C.c_void_p), a.size))
        self.check(self.lib.mph_runner_finalize(self.h))

    def close(self):
        if self.h and self.owned:
            self.lib.mph_runner_free(self.h)
        self.h = None

    def reserve_request(self, id, tokens):
        return ADMISSION[self.check(self.lib.mph_runner_reserve(self.h, _ids(id), C.c_size_t(tokens)))]

    def release_reservation(self, id):
        self.lib.mph_runner_release_reservation(self.h, _ids(id))

    def create(self, id):
        self.check(self.lib.mph_runner_create(self.h, _ids(id)))

    def fork_sequence(self, source, target):
        self.check(self.lib.mph_runner_fork(self.h, _ids(source), _ids(target)))

    def reuse_prefix(self, id, prompt):
        a, p, n = _toks(prompt)
        return self.check(self.lib.mph_runner_reuse_prefix(self.h, _ids(id), p, n))

    def cache_prefix(self, id):
        self.check(self.lib.mph_runner_cache_prefix(self.h, _ids(id)))

    def clear_prefix_cache(self):
        self.check(self.lib.mph_runner_clear_prefix_cache(self.h))

    def append(self, id, tokens):
        a, p, n = _toks(tokens)
        logits = np.empty(self.vocabulary, dtype=np.float32)
        self.check(self.lib.mph_runner_append(self.h, _ids(id), p, n, logits.ctypes.data_as(C.c_void_p)))
        return logits

    def release(self, id):
        self.check(self.lib.mph_runner_release(self.h, _ids(id)))

    def clear(self):
        self.check(self.lib.mph_runner_clear(self.h))

    def stats(self):
        out = (C.c_size_t * 25)()
        self.lib.mph_runner_stats(self.h, out)
        return dict(zip(RUNNER_STATS_FIELDS, list(out)))

    def cost_stats(self):
        out = (C.c_uint64 * 8)()
        self.lib.mph_runner_cost_stats(self.h, out)
        return dict(zip(COST_FIELDS, list(out)))

    def set_cost_timing(self, enabled):
        self.lib.mph_runner_set_cost_timing(self.h, int(bool(enabled)))

    def context_limit(self):
        return self.lib.mph_runner_context_limit(self.h)

    def sequence(self, id):
        used = C.c_int32()
        blocks = (C.c_int32 * 65536)()
        n = self.check(self.lib.mph_runner_sequence(self.h, _ids(id), C.byref(used), blocks, 65536))
        return used.value, list(blocks[:n])

    def script(self, id, tokens):
        a, p, n = _toks(tokens)
        self.check(self.lib.mph_runner_script(self.h, _ids(id), p, n))

    def poison(self, token):
        self.check(self.lib.mph_runner_poison(self.h, int(token)))

    def regions(self):
        cap = 1 << 16
        out = (C.c_size_t * (5 * cap))()
        n = self.check(self.lib.mph_runner_regions(self.h, out, cap))
        return [tuple(out[5 * i:5 * i + 5]) for i in range(n)]


class Engine(_Base):
    """The Engine; takes ownership of ``runner`` (the runner handle stays usable
    for script()/poison() on a scripted runner but must not be freed)."""

    def __init__(self, runner: Runner, max_batch, token_budget, prefill_chunk, context):
        super().__init__()
        h = self.lib.mph_engine_new(runner.h, max_batch, token_budget, prefill_chunk, context)
        if not h:
            raise HostError(-1, self.error())
        runner.owned = False
        self.runner = runner
        self.h = _vp(h)

    def close(self):
        if self.h:
            self.lib.mph_engine_free(self.h)
            self.h = None

    def submit(self, id, prompt, max_new_tokens, eos=None):
        a, p, n = _toks(prompt)
        self.check(self.lib.mph_engine_submit(self.h, _ids(id), p, n, max_new_tokens, -1 if eos is None else int(eos)))

    def serve(self, text: str, capacity: int = 1 << 24) -> str:
        """Worker protocol v3 over this engine: the response lines to `text`'s
        commands (served once; a response longer than `capacity` raises)."""
        self.lib.mph_engine_serve.restype = C.c_long
        self.lib.mph_engine_serve.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_long]
        buf = C.create_string_buffer(capacity)
        n = self.check(self.lib.mph_engine_serve(self.h, text.encode(), buf, capacity))
        if n >= capacity:
            raise HostError(-6, f"protocol response of {n} bytes exceeds the {capacity}-byte buffer")
        return buf.raw[:n].decode()

    def step(self) -> bool:
        return bool(self.check(self.lib.mph_engine_step(self.h)))

    def poll_events(self):
        cap = 1 << 22
        buf = C.create_string_buffer(cap)
        n = self.lib.mph_engine_poll(self.h, buf, cap)
        if n >= cap:
            raise RuntimeError("event text larger than buffer")
        events = []
        for line in buf.value.decode().split("\n"):
            if not line:
                continue
            rid, tok, reason, err = line.split("\t", 3)
            events.append((rid, None if int(tok) < 0 else int(tok), None if int(reason) < 0 else int(reason), err))
        return events

    def poll_compact(self, capacity=1 << 16):
        """The pending events as three int32 arrays (request index, token or -1,
        finish reason or -1). The receive buffers are allocated once per engine and
        capacity; the returned arrays are copies."""
        bufs = getattr(self, "_poll_bufs", None)
        if bufs is None or bufs[0] != capacity:
            arrays = [np.empty(capacity, dtype=np.int32) for _ in range(3)]
            bufs = self._poll_bufs = (capacity, arrays, [C.c_void_p(a.ctypes.data) for a in arrays])
        _, (req, tok, rea), ptrs = bufs
        n = self.lib.mph_engine_poll_compact(self.h, ptrs[0], ptrs[1], ptrs[2], capacity)
        if n > capacity:
            raise RuntimeError("more events than capacity")
        return req[:n].copy(), tok[:n].copy(), rea[:n].copy()

    def cancel(self, id):
        self.check(self.lib.mph_engine_cancel(self.h, _ids(id)))

    def shutdown(self):
        self.check(self.lib.mph_engine_shutdown(self.h))

    def idle(self):
        return bool(self.lib.mph_engine_idle(self.h))

    def failed(self):
        return bool(self.lib.mph_engine_failed(self.h))

    def last_step_stats(self):
        out = (C.c_size_t * 3)()
        self.lib.mph_engine_step_stats(self.h, out)
        return dict(zip(("prefix_reused_tokens", "prefill_tokens", "decode_tokens"), list(out)))

    def runner_stats(self):
        out = (C.c_size_t * 25)()
        self.lib.mph_engine_runner_stats(self.h, out)
        return dict(zip(RUNNER_STATS_FIELDS, list(out)))

    def cost_stats(self):
        out = (C.c_uint64 * 8)()
        self.lib.mph_engine_cost_stats(self.h, out)
        return dict(zip(COST_FIELDS, list(out)))

    def sequence(self, id):
        used = C.c_int32()
        blocks = (C.c_int32 * 65536)()
        rc = self.lib.mph_engine_sequence(self.h, _ids(id), C.byref(used), blocks, 65536)
        if rc < 0:
            return None
        return used.value, list(blocks[:rc])

    def flushes(self):
        f, h = C.c_size_t(), C.c_size_t()
        self.lib.mph_engine_flushes(self.h, C.byref(f), C.byref(h))
        return f.value, h.value

    def script(self, id, tokens):
        self.runner.script(id, tokens)

    def capture_logits(self, on: bool) -> None:
        """While on, every device forward also keeps the logits of its appends
        (parity checks of batched runs; see logits())."""
        self.lib.mph_engine_capture_logits.argtypes = [C.c_void_p, C.c_int32]
        self.check(self.lib.mph_engine_capture_logits(self.h, int(bool(on))))

    def logits(self, id):
        """The latest captured logits of request `id`, or None."""
        self.lib.mph_engine_logits.restype = C.c_long
        self.lib.mph_engine_logits.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_long]
        n = self.lib.mph_engine_logits(self.h, _ids(id), None, 0)
        if n < 0:
            return None
        out = np.empty(n, dtype=np.float32)
        self.lib.mph_engine_logits(self.h, _ids(id), out.ctypes.data_as(C.c_void_p), n)
        return out

    def device(self):
        """A device.ContextView of the engine's B200 context (None for other runners)."""
        h = self.lib.mph_engine_device(self.h)
        return _device.ContextView(h) if h else None
