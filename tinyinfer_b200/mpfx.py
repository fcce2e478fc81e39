"""MPFX0001 model files (the reference's weight format, miniprefix/src/model/
model.cpp:20-56; writer miniprefix/tools/prepare_model.py:34-50).

`write` produces the format from a ModelConfig and a name -> array dict (2-D
linears [in][out], as synthetic.random_weights returns them); `read` and
`read_config` go through the host library's reader, which applies the reference
loader's checks and messages. Runner.b200_from_file loads a file straight into a
B200 runner.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import device as _device
from .synthetic import ModelConfig


def tensor_names(cfg: ModelConfig) -> list[str]:
    """Every tensor an MPFX0001 file of this config holds (model.cpp:31-41)."""
    names = ["model.embed_tokens.weight", "model.norm.weight"]
    if not cfg.tied:
        names.append("lm_head.weight")
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}."
        names += [p + s for s in ("input_layernorm.weight", "post_attention_layernorm.weight",
                                  "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                  "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                                  "mlp.down_proj.weight")]
    return names


def write(path: str, cfg: ModelConfig, weights: dict, order: list[str] | None = None) -> None:
    """Writes an MPFX0001 file; tensors in `order` (default tensor_names(cfg))."""
    names = order if order is not None else tensor_names(cfg)
    with open(path, "wb") as f:
        f.write(b"MPFX0001")
        f.write(struct.pack("<8i2fII", cfg.layers, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads,
                            cfg.vocabulary, cfg.context, cfg.eos, cfg.rms_epsilon, cfg.rope_theta, int(cfg.tied),
                            len(names)))
        for name in names:
            a = np.ascontiguousarray(weights[name], dtype="<f4")
            encoded = name.encode()
            f.write(struct.pack("<I", len(encoded)) + encoded)
            f.write(struct.pack("<I", a.ndim))
            f.write(struct.pack("<" + "i" * a.ndim, *a.shape))
            f.write(struct.pack("<Q", a.nbytes))
            f.write(a.tobytes())


_SINK = C.CFUNCTYPE(C.c_int, C.c_char_p, C.POINTER(C.c_float), C.c_uint64, C.c_void_p)


def _lib():
    from . import host

    lib = host.library()
    lib.mph_mpfx_config.argtypes = [C.c_char_p, C.POINTER(_device.ModelConfigC)]
    lib.mph_mpfx_read.argtypes = [C.c_char_p, C.POINTER(_device.ModelConfigC), _SINK, C.c_void_p]
    return lib


def _config(m: _device.ModelConfigC) -> ModelConfig:
    return ModelConfig(layers=m.layers, hidden=m.hidden, intermediate=m.intermediate, heads=m.heads,
                       kv_heads=m.kv_heads, vocabulary=m.vocabulary, context=m.context, eos=m.eos,
                       rms_epsilon=m.rms_epsilon, rope_theta=m.rope_theta, tied=bool(m.tied))


def _check(lib, rc):
    from .host import HostError

    if rc < 0:
        raise HostError(rc, lib.mph_last_error().decode())


def read_config(path: str) -> ModelConfig:
    lib = _lib()
    m = _device.ModelConfigC()
    _check(lib, lib.mph_mpfx_config(path.encode(), C.byref(m)))
    return _config(m)


def read(path: str) -> tuple[ModelConfig, dict]:
    """Config and tensors (flat float32 arrays, file order) through the host reader."""
    lib = _lib()
    out = {}

    def sink(name, data, elements, user):
        out[name.decode()] = np.ctypeslib.as_array(data, shape=(int(elements),)).copy()
        return 0

    cb = _SINK(sink)
    m = _device.ModelConfigC()
    _check(lib, lib.mph_mpfx_read(path.encode(), C.byref(m), cb, None))
    return _config(m), out
