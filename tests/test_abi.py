"""The C-ABI library builds for sm_100a, loads, and exports every entry point
that include/*.h declares (CPU only: no compute call is made)."""

import ctypes
import glob
import os
import re
import subprocess

from conftest import ROOT


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(sr_[A-Za-z0-9_]+)\s*\(", text, re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "sr_step" in names and "sr_sample" in names and "sr_model_create" in names
    from sr_go_tranformer_b200 import _abi
    assert set(names) == set(_abi.EXPORTED), set(names) ^ set(_abi.EXPORTED)


def test_library_exports_every_declared_symbol(srlib):
    from sr_go_tranformer_b200 import _abi
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    for name in declared_functions():
        assert name in exported, name
        assert getattr(srlib, name) is not None


def test_error_path_without_device(srlib):
    """A null argument is rejected before any CUDA call."""
    from sr_go_tranformer_b200 import _abi
    rc = srlib.sr_model_create(None, 0, None)
    assert rc == _abi.SR_EINVAL
    assert b"null" in srlib.sr_last_error()
    assert b"sm_100a" in srlib.sr_version()
    assert isinstance(ctypes.c_int(rc).value, int)


def test_null_model_rejected_before_any_device_call(srlib):
    """Every model entry point added beside the step (mode, code cache, split
    steps, single projection, sampler over host logits) refuses a null model
    with SR_EINVAL and a message, touching no device."""
    from sr_go_tranformer_b200 import _abi
    out = ctypes.c_int32()
    calls = [
        lambda: srlib.sr_model_set_mode(None, 1),
        lambda: srlib.sr_model_set_code_cache(None, 1),
        lambda: srlib.sr_model_code_cache(None, ctypes.byref(out)),
        lambda: srlib.sr_model_set_split(None, 1),
        lambda: srlib.sr_linear(None, 0, 1, None, None),
        lambda: srlib.sr_sample_logits(None, 1, 8, None, None, None, None, None, -1, None),
    ]
    for call in calls:
        assert call() == _abi.SR_EINVAL
        assert b"null" in srlib.sr_last_error()
