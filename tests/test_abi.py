"""CPU checks of the C ABI boundary: the library loads and exports every
symbol include/orx.h declares (no compute calls without a GPU)."""
import ctypes
import os
import subprocess

import pytest

from orator_b200 import _lib


def _ensure_built():
    if not os.path.exists(_lib.LIB_PATH):
        from orator_b200.build import build
        build()


def test_header_symbols_bound():
    declared = set(_lib.header_symbols())
    assert declared, "no declarations parsed"
    missing = declared - set(_lib._SIGS)
    assert not missing, f"header functions without a binding: {missing}"


def test_library_exports_all_header_symbols():
    _ensure_built()
    L = ctypes.CDLL(_lib.LIB_PATH)
    for name in _lib.header_symbols():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(_lib.header_symbols()) <= exported


def test_version_and_defaults():
    _ensure_built()
    L = _lib.lib()
    assert L.orx_version() >= 1
    cfg = _lib.Config()
    L.orx_config_default(ctypes.byref(cfg))
    assert (cfg.hidden_size, cfg.num_layers, cfg.vocab_size, cfg.max_seq_len) == (2048, 28, 151936, 2048)
    assert cfg.rope_theta == 1e6


def test_create_rejects_other_geometry():
    """Argument validation runs before any device work."""
    _ensure_built()
    cfg = _lib.Config()
    _lib.lib().orx_config_default(ctypes.byref(cfg))
    cfg.hidden_size = 1024
    h = ctypes.c_void_p()
    with pytest.raises(_lib.OrxError) as e:
        _lib.call("orx_decoder_create", ctypes.byref(cfg), ctypes.byref(h))
    assert e.value.code == 1


def test_null_arguments_rejected():
    _ensure_built()
    with pytest.raises(_lib.OrxError):
        _lib.call("orx_decoder_create", None, None)
