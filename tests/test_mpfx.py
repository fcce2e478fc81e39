"""MPFX0001 model files: the host reader vs the reference loader (ModelWeights::load,
miniprefix/src/model/model.cpp:20-56), on well-formed files and on every failure the
reference checks for, in its order. Both must accept the same files with the same
config and tensors, and reject malformed ones with the same message.
"""
import os
import struct

import numpy as np
import pytest

from tinyinfer_b200 import mpfx
from tinyinfer_b200.host import HostError
from tinyinfer_b200.synthetic import ModelConfig, random_weights

SMALL = ModelConfig(layers=2, hidden=64, intermediate=96, heads=4, kv_heads=2, vocabulary=50, context=40, eos=3,
                    rms_epsilon=1e-5, rope_theta=1e4, tied=True)


def small_weights(cfg, seed=3):
    return random_weights(cfg, seed=seed)


def raw_file(path, cfg, weights, *, magic=b"MPFX0001", tied=None, count=None, names=None, patch=None, tail=b""):
    """Writes an MPFX0001 file with optional defects. patch(name, fields) may edit
    the per-tensor fields dict {name_bytes, rank, dims, nbytes, data} before it is
    written (returning None drops the rest of the file after the header)."""
    names = names if names is not None else mpfx.tensor_names(cfg)
    with open(path, "wb") as f:
        f.write(magic)
        f.write(struct.pack("<8i2f", cfg.layers, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads,
                            cfg.vocabulary, cfg.context, cfg.eos, cfg.rms_epsilon, cfg.rope_theta))
        f.write(struct.pack("<I", int(cfg.tied) if tied is None else tied))
        f.write(struct.pack("<I", len(names) if count is None else count))
        for name in names:
            a = np.ascontiguousarray(weights[name], dtype="<f4")
            fields = {"name": name.encode(), "rank": a.ndim, "dims": list(a.shape), "nbytes": a.nbytes,
                      "data": a.tobytes()}
            if patch:
                fields = patch(name, fields)
                if fields is None:
                    break
            f.write(struct.pack("<I", len(fields["name"])) + fields["name"])
            f.write(struct.pack("<I", fields["rank"]))
            f.write(struct.pack("<" + "i" * len(fields["dims"]), *fields["dims"]))
            f.write(struct.pack("<Q", fields["nbytes"]))
            f.write(fields["data"])
        f.write(tail)


def ours(path):
    try:
        return "ok", mpfx.read(path)
    except HostError as e:
        return "err", e.message


def theirs(ref, path):
    from oracle.oracle import RefError

    try:
        return "ok", ref.load_mpfx(path)
    except RefError as e:
        return "err", e.message


def message(result):
    return result[1] if result[0] == "err" else None


@pytest.mark.parametrize("tied", [True, False])
def test_round_trip_matches_reference(built, ref, tmp_path, tied):
    cfg = ModelConfig(**{**SMALL.__dict__, "tied": tied})
    w = small_weights(cfg)
    path = str(tmp_path / "m.mpfx")
    mpfx.write(path, cfg, w)
    got_cfg, got = mpfx.read(path)
    ref_cfg, ref_t = ref.load_mpfx(path)
    for c in (got_cfg, ref_cfg):
        assert (c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.vocabulary, c.context, c.eos, c.tied) == \
            (cfg.layers, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads, cfg.vocabulary, cfg.context, cfg.eos,
             cfg.tied)
        assert np.float32(c.rms_epsilon) == np.float32(cfg.rms_epsilon)
        assert np.float32(c.rope_theta) == np.float32(cfg.rope_theta)
    assert list(got) == mpfx.tensor_names(cfg)  # file order
    assert sorted(got) == sorted(ref_t)
    for name, a in got.items():
        assert np.array_equal(a, np.asarray(w[name], dtype=np.float32).reshape(-1)), name
        assert np.array_equal(a, ref_t[name]), name
    assert mpfx.read_config(path).layers == cfg.layers


def test_any_tensor_order(built, ref, tmp_path):
    w = small_weights(SMALL)
    names = mpfx.tensor_names(SMALL)[::-1]
    path = str(tmp_path / "rev.mpfx")
    mpfx.write(path, SMALL, w, order=names)
    assert list(mpfx.read(path)[1]) == names
    assert sorted(ref.load_mpfx(path)[1]) == sorted(names)


def _defects(cfg, w):
    """(label, raw_file keyword arguments) for each check of the reference loader."""
    first = mpfx.tensor_names(cfg)[0]
    q0 = "model.layers.0.self_attn.q_proj.weight"

    def at(target, **edits):
        def patch(name, fields):
            if name == target:
                fields = {**fields, **edits}
            return fields
        return patch

    nan = np.asarray(w[q0], dtype="<f4").copy()
    nan.reshape(-1)[5] = np.nan
    return [
        ("magic", {"magic": b"MPFX0002"}),
        ("tied flag", {"tied": 2}),
        ("invalid config", {"cfg": ModelConfig(**{**cfg.__dict__, "heads": 3})}),
        ("count", {"count": len(mpfx.tensor_names(cfg)) + 1}),
        ("empty name", {"patch": at(first, name=b"")}),
        ("long name", {"patch": at(first, name=b"x" * 257)}),
        ("unknown name", {"patch": at(first, name=b"model.unknown.weight")}),
        ("duplicate", {"names": [first, first] + mpfx.tensor_names(cfg)[2:]}),
        ("rank", {"patch": at(q0, rank=1, dims=[cfg.hidden])}),
        ("shape", {"patch": at(q0, dims=[cfg.hidden, cfg.hidden - 1])}),
        ("bytes", {"patch": at(q0, nbytes=cfg.hidden * cfg.hidden * 4 + 4)}),
        ("nonfinite", {"patch": at(q0, data=nan.tobytes())}),
        ("trailing", {"tail": b"\x00"}),
        ("truncated tensor", {"truncate_data": (q0, 100)}),
    ]


def test_malformed_files_fail_like_reference(built, ref, tmp_path):
    w = small_weights(SMALL)
    seen = set()
    for label, kw in _defects(SMALL, w):
        path = str(tmp_path / (label.replace(" ", "_") + ".mpfx"))
        cfg = kw.pop("cfg", SMALL)
        trunc = kw.pop("truncate_data", None)
        raw_file(path, cfg, w, **kw)
        if trunc:
            # cut the file in the middle of the tensor's data
            mpfx.write(path, cfg, w)
            names = mpfx.tensor_names(cfg)
            offset = 8 + 44 + 4
            for name in names:
                a = np.asarray(w[name], dtype=np.float32)
                offset += 4 + len(name.encode()) + 4 + 4 * a.ndim + 8
                if name == trunc[0]:
                    break
                offset += a.nbytes
            with open(path, "r+b") as f:
                f.truncate(offset + trunc[1])
        a, b = ours(path), theirs(ref, path)
        assert a[0] == "err" and b[0] == "err", (label, a[0], b[0])
        assert message(a) == message(b), (label, message(a), message(b))
        seen.add(message(b))
    # truncated header and name, a missing file
    for label, data in (("short header", b"MPFX0001" + b"\x01\x00"), ("short name", None)):
        path = str(tmp_path / (label.replace(" ", "_") + ".mpfx"))
        if data is not None:
            open(path, "wb").write(data)
        else:
            mpfx.write(path, SMALL, w)
            with open(path, "r+b") as f:
                f.truncate(8 + 44 + 4 + 4 + 5)
        a, b = ours(path), theirs(ref, path)
        assert message(a) == message(b) and a[0] == "err", (label, message(a), message(b))
        seen.add(message(b))
    missing = str(tmp_path / "absent.mpfx")
    assert message(ours(missing)) == message(theirs(ref, missing)) == f"cannot open model: {missing}"
    assert {"invalid model format", "invalid tied flag", "unsupported/invalid Llama configuration",
            "model tensor count mismatch", "invalid tensor name", "tensor rank mismatch", "invalid tensor bytes",
            "nonfinite weights", "trailing model data", "truncated model", "truncated name"} <= seen, seen
    # a file cut inside a tensor's data fails the size check first (model.cpp:48),
    # so "truncated tensor" needs a file that shrinks while it is read


def test_runner_from_missing_file_reports(built):
    from tinyinfer_b200.host import Runner

    with pytest.raises(HostError) as e:
        Runner.b200_from_file(os.path.join("/nonexistent", "m.mpfx"), context=16)
    assert "cannot open model" in str(e.value)
