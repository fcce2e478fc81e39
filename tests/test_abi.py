"""The C-ABI libraries load and export every function the public headers declare (no GPU calls)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mp[a-z_]*)\s*\(", text)))


@pytest.mark.parametrize("header,lib", [("miniprefix_b200.h", "libmpb200.so"),
                                        ("miniprefix_b200_host.h", "libmpb200_host.so")])
def test_exports(built, header, lib):
    path = os.path.join(ROOT, "include", header)
    if not os.path.exists(path):
        pytest.skip(f"{header} not present")
    names = declared(header)
    assert names, "header declares no functions"
    so = ctypes.CDLL(os.path.join(built, lib))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, f"{lib} misses {missing}"


def test_device_library_rejects_bad_config_without_gpu(built):
    """mp_create validates the geometry before touching a device."""
    from tinyinfer_b200 import device
    from tinyinfer_b200.synthetic import ModelConfig

    bad = ModelConfig(heads=8, kv_heads=2, hidden=512)
    with pytest.raises(device.DeviceError) as e:
        device.DeviceContext(bad)
    assert e.value.code == device.MP_ERR_UNSUPPORTED
