"""ctypes loaders for the CPU oracles -- TEST INFRASTRUCTURE ONLY.

Two checkers, both built by oracle/Makefile:
  * ``Oracle``   -- libmporacle.so, the plain-C restatement of the reference CPU
                    runner's arithmetic (mp_oracle.c).
  * ``RefLib``   -- _ref/libmpref.so, the unmodified reference MiniPrefix CPU
                    engine (CpuRunner, KVManager, Engine) behind ref_shim.cpp.
Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
import this module. The product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference checkout whose sources build _ref/: MINIPREFIX_REFERENCE when set,
# else a directory named `reference` beside this repository (oracle/Makefile uses
# the same rule).
REFERENCE = os.environ.get("MINIPREFIX_REFERENCE",
                           os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
ORACLE_SO = os.path.join(HERE, "libmporacle.so")
REF_SO = os.path.join(HERE, "_ref", "libmpref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build_oracle() -> None:
    """Compile libmporacle.so (gcc only; no reference sources needed)."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)


DROPIN_TEST = os.path.join(HERE, "_ref", "cow_test_b200")


def build_ref() -> bool:
    """Compile _ref/libmpref.so (the reference CPU engine) and, once the product
    libraries exist, _ref/cow_test_b200 (the reference's cow_test.cpp on the B200
    drop-in runner) when the reference sources are present."""
    if not os.path.isdir(REFERENCE):
        return os.path.exists(REF_SO)
    targets = ["ref"]
    if os.path.exists(os.path.join(os.path.dirname(HERE), "tinyinfer_b200", "libmpb200_host.so")):
        targets.append("dropin")
    subprocess.run(["make", "-s", "-j8", "-C", HERE, *targets, f"MINIPREFIX_REFERENCE={REFERENCE}"], check=True)
    return True


class _Config(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("intermediate", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("vocabulary", C.c_int), ("rms_epsilon", C.c_float),
                ("rope_theta", C.c_float), ("tied", C.c_int), ("block_tokens", C.c_int)]


class _Weights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("lm_head", C.c_void_p)] + [
        (n, C.POINTER(C.c_void_p)) for n in ("input_norm", "post_norm", "q", "k", "v", "o", "gate", "up", "down")]


class Oracle:
    """The C restatement. Holds a model (config + weights dict) and runs appends."""

    def __init__(self, config, weights: dict, block_tokens: int = 16):
        if not os.path.exists(ORACLE_SO):
            build_oracle()
        self.lib = C.CDLL(ORACLE_SO)
        self.lib.oracle_append.restype = C.c_int
        self.config = config
        self.block_tokens = block_tokens
        self._keep = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
        c = config
        self._cfg = _Config(c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.vocabulary,
                            c.rms_epsilon, c.rope_theta, int(c.tied), block_tokens)
        ptr = lambda a: a.ctypes.data_as(C.c_void_p)
        arrays = {}
        for key, suffix in [("input_norm", "input_layernorm.weight"), ("post_norm", "post_attention_layernorm.weight"),
                            ("q", "self_attn.q_proj.weight"), ("k", "self_attn.k_proj.weight"),
                            ("v", "self_attn.v_proj.weight"), ("o", "self_attn.o_proj.weight"),
                            ("gate", "mlp.gate_proj.weight"), ("up", "mlp.up_proj.weight"),
                            ("down", "mlp.down_proj.weight")]:
            arr = (C.c_void_p * c.layers)(*[ptr(self._keep[f"model.layers.{l}.{suffix}"]) for l in range(c.layers)])
            arrays[key] = arr
        self._arrays = arrays
        self._w = _Weights(ptr(self._keep["model.embed_tokens.weight"]), ptr(self._keep["model.norm.weight"]),
                           ptr(self._keep["lm_head.weight"]) if not c.tied else None,
                           *[C.cast(arrays[k], C.POINTER(C.c_void_p)) for k in
                             ("input_norm", "post_norm", "q", "k", "v", "o", "gate", "up", "down")])

    def new_pools(self, max_blocks: int) -> tuple[np.ndarray, np.ndarray]:
        n = max_blocks * self.config.layers * self.block_tokens * self.config.kv_width
        return np.zeros(n, dtype=np.float32), np.zeros(n, dtype=np.float32)

    def append(self, keys, values, blocks, used: int, tokens) -> tuple[np.ndarray, bool]:
        """Logits of the last appended row; writes K/V rows. Returns (logits, finite)."""
        blocks = np.ascontiguousarray(blocks, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.config.vocabulary, dtype=np.float32)
        bad = self.lib.oracle_append(C.byref(self._cfg), C.byref(self._w), keys.ctypes.data_as(C.c_void_p),
                                     values.ctypes.data_as(C.c_void_p), blocks.ctypes.data_as(C.c_void_p),
                                     C.c_int(used), tokens.ctypes.data_as(C.c_void_p), C.c_int(len(tokens)),
                                     logits.ctypes.data_as(C.c_void_p))
        return logits, bad == 0

    @staticmethod
    def decode_attention(q, lengths, tables, keys, values, heads, kv_heads, dim, block_tokens):
        """Paged decode attention operator, one query row per sequence (one-layer pool)."""
        if not os.path.exists(ORACLE_SO):
            build_oracle()
        lib = C.CDLL(ORACLE_SO)
        q = np.ascontiguousarray(q, dtype=np.float32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        tables = np.ascontiguousarray(tables, dtype=np.int32)
        out = np.empty_like(q)
        lib.oracle_decode_attention(q.ctypes.data_as(C.c_void_p), C.c_int(len(lengths)),
                                    lengths.ctypes.data_as(C.c_void_p), tables.ctypes.data_as(C.c_void_p),
                                    C.c_int(tables.shape[1]), keys.ctypes.data_as(C.c_void_p),
                                    values.ctypes.data_as(C.c_void_p), C.c_int(heads), C.c_int(kv_heads),
                                    C.c_int(dim), C.c_int(block_tokens), out.ctypes.data_as(C.c_void_p))
        return out


class RefError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class RefLib:
    """Thin ctypes view of _ref/libmpref.so (the reference engine)."""

    def __init__(self):
        if not os.path.exists(REF_SO) and not build_ref():
            raise FileNotFoundError("reference engine library not built (oracle/_ref/libmpref.so)")
        lib = C.CDLL(REF_SO)
        lib.ref_last_error.restype = C.c_char_p
        for name in ("ref_weights_new", "ref_cpu_runner_new", "ref_scripted_runner_new", "ref_kv_new",
                     "ref_engine_new"):
            getattr(lib, name).restype = C.c_void_p
        lib.ref_weights_new.argtypes = [C.c_int] * 8 + [C.c_float, C.c_float, C.c_int]
        lib.ref_weights_load.restype = C.c_void_p
        lib.ref_weights_load.argtypes = [C.c_char_p]
        lib.ref_weights_config.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_float)]
        lib.ref_weights_tensor.restype = C.c_long
        lib.ref_weights_tensor.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_long]
        lib.ref_weights_count.restype = C.c_long
        lib.ref_weights_count.argtypes = [C.c_void_p]
        lib.ref_weights_free.argtypes = [C.c_void_p]
        lib.ref_weights_put.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int, C.c_void_p]
        lib.ref_cpu_runner_new.argtypes = [C.c_void_p] + [C.c_int] * 4
        lib.ref_scripted_runner_new.argtypes = [C.c_int] * 7
        lib.ref_kv_new.argtypes = [C.c_int] * 7
        lib.ref_engine_new.argtypes = [C.c_void_p] + [C.c_int] * 4
        for name in ("ref_runner_reuse_prefix", "ref_kv_reuse_prefix", "ref_kv_offset", "ref_engine_poll",
                     "ref_scripted_regions", "ref_engine_regions"):
            getattr(lib, name).restype = C.c_long
        for name in ("ref_runner_reserve", "ref_kv_reserve"):
            getattr(lib, name).argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        self.lib = lib

    def error(self) -> str:
        return self.lib.ref_last_error().decode()

    def check(self, rc: int) -> int:
        if rc < 0:
            raise RefError(rc, self.error())
        return rc

    def weights(self, config, weights: dict):
        c = config
        h = self.lib.ref_weights_new(c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.vocabulary,
                                     c.context, c.eos, c.rms_epsilon, c.rope_theta, int(c.tied))
        if not h:
            raise RefError(-1, self.error())
        for name, arr in weights.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            dims = (C.c_long * a.ndim)(*a.shape)
            self.check(self.lib.ref_weights_put(C.c_void_p(h), name.encode(), a.ctypes.data_as(C.c_void_p),
                                                a.ndim, dims))
        return h

    def load_mpfx(self, path: str):
        """The reference loader on an MPFX0001 file: (config ints, (eps, theta),
        {name: flat float32 array}); RefError with its message on failure."""
        h = self.lib.ref_weights_load(path.encode())
        if not h:
            raise RefError(-4, self.error())
        try:
            ints = (C.c_int * 9)()
            floats = (C.c_float * 2)()
            self.lib.ref_weights_config(C.c_void_p(h), ints, floats)
            from tinyinfer_b200 import mpfx
            from tinyinfer_b200.synthetic import ModelConfig

            cfg = ModelConfig(*list(ints)[:8], rms_epsilon=floats[0], rope_theta=floats[1], tied=bool(ints[8]))
            out = {}
            for name in mpfx.tensor_names(cfg):
                n = self.lib.ref_weights_tensor(C.c_void_p(h), name.encode(), None, 0)
                a = np.empty(n, dtype=np.float32)
                self.lib.ref_weights_tensor(C.c_void_p(h), name.encode(), a.ctypes.data_as(C.c_void_p), n)
                out[name] = a
            assert self.lib.ref_weights_count(C.c_void_p(h)) == len(out)
            return cfg, out
        finally:
            self.lib.ref_weights_free(C.c_void_p(h))


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
ADMISSION = ("Ready", "Wait", "Impossible")


def _ids(x) -> bytes:
    return x.encode() if isinstance(x, str) else x


def _toks(tokens):
    a = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
    return a, a.ctypes.data_as(C.c_void_p), len(a)


class RefRunner:
    """The reference ModelRunner (CpuRunner, or the scripted runner over a real
    KVManager) driven through ref_shim.cpp. Methods mirror
    miniprefix/include/miniprefix/model.h:35-58."""

    def __init__(self, ref: RefLib, handle, vocabulary: int, scripted: bool = False):
        self.ref, self.h, self.vocabulary, self.scripted = ref, C.c_void_p(handle), vocabulary, scripted

    @classmethod
    def cpu(cls, ref: RefLib, config, weights: dict, context: int, block_tokens=16, max_blocks=128, prefix_blocks=0):
        w = ref.weights(config, weights)
        h = ref.lib.ref_cpu_runner_new(C.c_void_p(w), context, block_tokens, max_blocks, prefix_blocks)
        ref.lib.ref_weights_free(C.c_void_p(w))
        if not h:
            raise RefError(-1, ref.error())
        return cls(ref, h, config.vocabulary)

    @classmethod
    def scripted_runner(cls, ref: RefLib, vocabulary, context, layers, width, block_tokens=16, max_blocks=128,
                        prefix_blocks=0):
        h = ref.lib.ref_scripted_runner_new(vocabulary, context, layers, width, block_tokens, max_blocks, prefix_blocks)
        if not h:
            raise RefError(-1, ref.error())
        return cls(ref, h, vocabulary, scripted=True)

    def close(self):
        if self.h:
            self.ref.lib.ref_runner_free(self.h)
            self.h = None

    def _c(self, rc):
        return self.ref.check(rc)

    def reserve_request(self, id, tokens):
        return ADMISSION[self._c(self.ref.lib.ref_runner_reserve(self.h, _ids(id), C.c_size_t(tokens)))]

    def release_reservation(self, id):
        self.ref.lib.ref_runner_release_reservation(self.h, _ids(id))

    def create(self, id):
        self._c(self.ref.lib.ref_runner_create(self.h, _ids(id)))

    def fork_sequence(self, source, target):
        self._c(self.ref.lib.ref_runner_fork(self.h, _ids(source), _ids(target)))

    def reuse_prefix(self, id, prompt):
        a, p, n = _toks(prompt)
        return self._c(self.ref.lib.ref_runner_reuse_prefix(self.h, _ids(id), p, n))

    def cache_prefix(self, id):
        self._c(self.ref.lib.ref_runner_cache_prefix(self.h, _ids(id)))

    def clear_prefix_cache(self):
        self._c(self.ref.lib.ref_runner_clear_prefix_cache(self.h))

    def append(self, id, tokens):
        a, p, n = _toks(tokens)
        logits = np.empty(self.vocabulary, dtype=np.float32)
        self._c(self.ref.lib.ref_runner_append(self.h, _ids(id), p, n, logits.ctypes.data_as(C.c_void_p)))
        return logits

    def release(self, id):
        self._c(self.ref.lib.ref_runner_release(self.h, _ids(id)))

    def clear(self):
        self._c(self.ref.lib.ref_runner_clear(self.h))

    def stats(self) -> dict:
        out = (C.c_size_t * 25)()
        self.ref.lib.ref_runner_stats(self.h, out)
        return dict(zip(RUNNER_STATS_FIELDS, list(out)))

    def cost_stats(self) -> dict:
        out = (C.c_uint64 * 8)()
        self.ref.lib.ref_runner_cost_stats(self.h, out)
        return dict(zip(COST_FIELDS, list(out)))

    def set_cost_timing(self, enabled: bool):
        self.ref.lib.ref_runner_set_cost_timing(self.h, int(bool(enabled)))

    def context_limit(self) -> int:
        return self.ref.lib.ref_runner_context_limit(self.h)

    # scripted-runner extras
    def script(self, id, tokens):
        a, p, n = _toks(tokens)
        self._c(self.ref.lib.ref_scripted_set(self.h, _ids(id), p, n))

    def poison(self, token):
        self._c(self.ref.lib.ref_scripted_poison(self.h, int(token)))

    def sequence(self, id):
        used = C.c_int()
        cap = 1 << 16
        blocks = (C.c_int * cap)()
        n = self._c(self.ref.lib.ref_scripted_sequence(self.h, _ids(id), C.byref(used), blocks, cap))
        return used.value, list(blocks[:n])

    def regions(self):
        cap = 1 << 16
        out = (C.c_size_t * (5 * cap))()
        n = self._c(self.ref.lib.ref_scripted_regions(self.h, out, cap))
        return [tuple(out[5 * i:5 * i + 5]) for i in range(n)]


class RefKV:
    """The reference KVManager (miniprefix/include/miniprefix/kv_manager.h:20-96)."""

    def __init__(self, ref: RefLib, block_tokens, max_blocks, prefix_blocks, layers, width, context, vocabulary):
        self.ref = ref
        h = ref.lib.ref_kv_new(block_tokens, max_blocks, prefix_blocks, layers, width, context, vocabulary)
        if not h:
            raise RefError(-1, ref.error())
        self.h = C.c_void_p(h)

    def close(self):
        if self.h:
            self.ref.lib.ref_kv_free(self.h)
            self.h = None

    def call(self, op: str, *args):
        """Run one KVManager operation; returns (code, result) without raising."""
        L = self.ref.lib
        if op == "reserve":
            rc = L.ref_kv_reserve(self.h, _ids(args[0]), C.c_size_t(args[1]))
            return rc, (ADMISSION[rc] if rc >= 0 else None)
        if op == "release_reservation":
            return L.ref_kv_release_reservation(self.h, _ids(args[0])), None
        if op == "create":
            return L.ref_kv_create(self.h, _ids(args[0])), None
        if op == "fork":
            return L.ref_kv_fork(self.h, _ids(args[0]), _ids(args[1])), None
        if op == "reuse_prefix":
            a, p, n = _toks(args[1])
            rc = L.ref_kv_reuse_prefix(self.h, _ids(args[0]), p, n)
            return (rc, rc) if rc < 0 else (0, rc)
        if op == "cache_prefix":
            return L.ref_kv_cache_prefix(self.h, _ids(args[0])), None
        if op == "clear_prefix_cache":
            return L.ref_kv_clear_prefix_cache(self.h), None
        if op == "append":
            a, p, n = _toks(args[1])
            tail = (C.c_long * 3)()
            region = (C.c_size_t * 5)()
            rc = L.ref_kv_append(self.h, _ids(args[0]), p, n, int(args[2]), tail, region)
            return rc, (tuple(tail), tuple(region) if tail[0] >= 0 and args[2] != 2 else None)
        if op == "reset_sequence":
            return L.ref_kv_reset_sequence(self.h, _ids(args[0])), None
        if op == "release":
            return L.ref_kv_release(self.h, _ids(args[0])), None
        if op == "clear":
            return L.ref_kv_clear(self.h), None
        raise ValueError(op)

    def stats(self) -> dict:
        out = (C.c_size_t * 16)()
        self.ref.lib.ref_kv_stats(self.h, out)
        return dict(zip(KV_STATS_FIELDS, list(out)))

    def sequence(self, id):
        used = C.c_int()
        cap = 1 << 16
        blocks = (C.c_int * cap)()
        rc = self.ref.lib.ref_kv_sequence(self.h, _ids(id), C.byref(used), blocks, cap)
        if rc < 0:
            return None
        return used.value, list(blocks[:rc])


class RefEngine:
    """The reference Engine (miniprefix/include/miniprefix/engine.h:10-37) over a RefRunner."""

    def __init__(self, runner: RefRunner, max_batch, token_budget, prefill_chunk, context):
        self.ref = runner.ref
        self.scripted = runner.scripted
        h = self.ref.lib.ref_engine_new(runner.h, max_batch, token_budget, prefill_chunk, context)
        if not h:
            raise RefError(-1, self.ref.error())
        self.h = C.c_void_p(h)

    def close(self):
        if self.h:
            self.ref.lib.ref_engine_free(self.h)
            self.h = None

    def submit(self, id, prompt, max_new_tokens, eos=None):
        a, p, n = _toks(prompt)
        self.ref.check(self.ref.lib.ref_engine_submit(self.h, _ids(id), p, n, C.c_uint(max_new_tokens),
                                                      -1 if eos is None else int(eos)))

    def step(self) -> bool:
        return bool(self.ref.check(self.ref.lib.ref_engine_step(self.h)))

    def serve(self, text: str, capacity: int = 1 << 24) -> str:
        """The reference worker protocol (apps/protocol/session.cpp) over this engine."""
        lib = self.ref.lib
        lib.ref_protocol_serve.restype = C.c_long
        lib.ref_protocol_serve.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_long]
        buf = C.create_string_buffer(capacity)
        n = lib.ref_protocol_serve(self.h, text.encode(), buf, capacity)
        assert n < capacity, "protocol response exceeds the buffer"
        return buf.raw[:n].decode()

    def poll_events(self):
        # ref_engine_poll drains on every call; call once with room for all text.
        return _parse_events(None, lambda buf, cap: self.ref.lib.ref_engine_poll(self.h, buf, cap))

    def cancel(self, id):
        self.ref.check(self.ref.lib.ref_engine_cancel(self.h, _ids(id)))

    def shutdown(self):
        self.ref.check(self.ref.lib.ref_engine_shutdown(self.h))

    def idle(self):
        return bool(self.ref.lib.ref_engine_idle(self.h))

    def failed(self):
        return bool(self.ref.lib.ref_engine_failed(self.h))

    def last_step_stats(self):
        out = (C.c_size_t * 3)()
        self.ref.lib.ref_engine_step_stats(self.h, out)
        return dict(zip(("prefix_reused_tokens", "prefill_tokens", "decode_tokens"), list(out)))

    def runner_stats(self):
        out = (C.c_size_t * 25)()
        self.ref.lib.ref_engine_runner_stats(self.h, out)
        return dict(zip(RUNNER_STATS_FIELDS, list(out)))

    def cost_stats(self):
        out = (C.c_uint64 * 8)()
        self.ref.lib.ref_engine_cost_stats(self.h, out)
        return dict(zip(COST_FIELDS, list(out)))

    def script(self, id, tokens):
        a, p, n = _toks(tokens)
        self.ref.check(self.ref.lib.ref_engine_script(self.h, _ids(id), p, n))

    def sequence(self, id):
        used = C.c_int()
        cap = 1 << 16
        blocks = (C.c_int * cap)()
        rc = self.ref.lib.ref_engine_sequence(self.h, _ids(id), C.byref(used), blocks, cap)
        if rc < 0:
            return None
        return used.value, list(blocks[:rc])

    def regions(self):
        cap = 1 << 16
        out = (C.c_size_t * (5 * cap))()
        n = self.ref.check(self.ref.lib.ref_engine_regions(self.h, out, cap))
        return [tuple(out[5 * i:5 * i + 5]) for i in range(n)]


def _parse_events(_need, fetch):
    cap = 1 << 22
    buf = C.create_string_buffer(cap)
    n = fetch(buf, cap)
    if n >= cap:
        raise RuntimeError("event text larger than buffer")
    events = []
    for line in buf.value.decode().split("\n"):
        if not line:
            continue
        rid, tok, reason, err = line.split("\t", 3)
        events.append((rid, None if int(tok) < 0 else int(tok), None if int(reason) < 0 else int(reason), err))
    return events


CACHE_STATS_FIELDS = ("size", "index_nodes", "key_token_bytes", "hits", "misses", "reused_tokens", "evictions",
                      "cache_only_blocks", "live_blocks", "peak_blocks", "free_blocks")


class RefCache:
    """The reference KvBlockPool + ExactPrefixCache over named sequences."""

    def __init__(self, ref: RefLib, block_tokens, max_blocks, prefix_blocks, layers=1, width=1):
        self.ref = ref
        ref.lib.ref_cache_new.restype = C.c_void_p
        ref.lib.ref_cache_reuse.restype = C.c_long
        h = ref.lib.ref_cache_new(block_tokens, max_blocks, prefix_blocks, layers, width)
        if not h:
            raise RefError(-1, ref.error())
        self.h = C.c_void_p(h)
        self.max_blocks = max_blocks

    def close(self):
        if self.h:
            self.ref.lib.ref_cache_free(self.h)
            self.h = None

    def append(self, seq, tokens):
        a, p, n = _toks(tokens)
        self.ref.check(self.ref.lib.ref_cache_append(self.h, _ids(seq), p, n))

    def publish(self, seq):
        self.ref.check(self.ref.lib.ref_cache_publish(self.h, _ids(seq)))

    def reuse(self, seq, prompt):
        a, p, n = _toks(prompt)
        return self.ref.check(self.ref.lib.ref_cache_reuse(self.h, _ids(seq), p, n))

    def release(self, seq):
        self.ref.check(self.ref.lib.ref_cache_release(self.h, _ids(seq)))

    def evict_one(self):
        return bool(self.ref.check(self.ref.lib.ref_cache_evict_one(self.h)))

    def clear(self):
        self.ref.lib.ref_cache_clear(self.h)

    def stats(self):
        out = (C.c_uint64 * 11)()
        self.ref.lib.ref_cache_stats(self.h, out)
        return dict(zip(CACHE_STATS_FIELDS, list(out)))

    def references(self):
        out = (C.c_uint64 * self.max_blocks)()
        self.ref.check(self.ref.lib.ref_cache_references(self.h, out, self.max_blocks))
        return list(out)

    def define(self, seq, used, tokens, blocks):
        """Set a sequence verbatim (no page accounting) to build malformed inputs."""
        a, p, n = _toks(tokens)
        b, q, m = _toks(blocks)
        self.ref.check(self.ref.lib.ref_cache_define(self.h, _ids(seq), int(used), p, n, q, m))

    def sequence(self, seq):
        used = C.c_int()
        blocks = (C.c_int * 65536)()
        toks = (C.c_int * 65536)()
        n = self.ref.check(self.ref.lib.ref_cache_sequence(self.h, _ids(seq), C.byref(used), blocks, 65536, toks, 65536))
        return used.value, list(blocks[:n]), list(toks[:used.value])
