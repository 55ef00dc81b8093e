"""The C-ABI library loads without a GPU and exports every entry point that
include/*.h declares; host-only helpers (registry ids, workspace sizes,
error mapping) behave like the reference."""

import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w \t\*]*?\b(oxc_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "oxc_rms_norm_fwd" in names and "oxc_layer_norm_bwd" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    from oxitorch_b200 import _native
    lib = _native.load(require_device=False)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding covers every declared entry point too
    unbound = [n for n in declared_functions() if n not in _native.SIGNATURES]
    assert not unbound, f"declared but not bound in _native.SIGNATURES: {unbound}"


def test_registry_ids_follow_reference_order():
    """Op ids are positions in ops.rs:55-202 / ReduceKind ops.rs:224-239."""
    from oxitorch_b200 import _native
    from oracle import oxiref
    lib = _native.load(require_device=False)
    for i, n in enumerate(oxiref.BINARY_OPS):
        assert lib.oxc_binary_op_id(n.encode()) == i
    for i, n in enumerate(oxiref.CMP_OPS):
        assert lib.oxc_cmp_op_id(n.encode()) == i
    for i, n in enumerate(oxiref.UNARY_OPS):
        assert lib.oxc_unary_op_id(n.encode()) == i
    for i, n in enumerate(oxiref.REDUCE_KINDS):
        assert lib.oxc_reduce_kind_id(n.encode()) == i
    assert lib.oxc_binary_op_id(b"frobnicate") == -1
    assert lib.oxc_unary_op_id(b"frob") == -1


def test_workspace_sizes_are_host_side():
    from oxitorch_b200 import _native
    lib = _native.load(require_device=False)
    assert lib.oxc_rms_norm_bwd_workspace_size(0, 4096) == 0
    assert lib.oxc_rms_norm_bwd_workspace_size(4096, 4096) % 16 == 0
    assert lib.oxc_layer_norm_bwd_workspace_size(16384, 4096) > 0


def test_status_to_exception_mapping():
    """crates/oxi-bindings/src/error.rs:22-32."""
    from oxitorch_b200 import _native as N
    N.load(require_device=False)
    for code, exc in [(N.ERR_INVALID_ARGUMENT, ValueError), (N.ERR_SHAPE_MISMATCH, ValueError),
                      (N.ERR_NOT_IMPLEMENTED, NotImplementedError),
                      (N.ERR_OUT_OF_BOUNDS, RuntimeError), (N.ERR_OTHER, RuntimeError),
                      (N.ERR_TIMEOUT, RuntimeError)]:
        with pytest.raises(exc):
            N.check(code, "probe")
    N.check(N.OK)


def test_cpu_tensors_are_rejected_before_any_launch():
    import torch
    from oxitorch_b200 import functional as F
    x = torch.zeros(2, 4)
    with pytest.raises(ValueError, match="CUDA"):
        F.rms_norm_fwd(x, torch.ones(4))


def test_struct_mirrors_match_the_header(tmp_path):
    """The ctypes mirrors of the ABI's structs have the header's size and
    field offsets (compiled with gcc against include/oxicuda.h)."""
    import shutil
    import subprocess
    from oxitorch_b200 import _native as N
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    checks = {
        "oxc_view": (N.View, ["data", "ndim", "shape", "strides"]),
        "oxc_emb_push": (N.EmbPush, ["world", "source", "cyclic", "local", "cap", "lo", "rows",
                                     "ids", "count"]),
        "oxc_emb_pull": (N.EmbPull, ["rows", "ids", "count"]),
    }
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "oxicuda.h"',
             "int main(void) {"]
    for cname, (_, fields) in checks.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), "-I", cuda_inc,
                           str(src), "-o", str(exe)])
    got = {}
    for line in subprocess.check_output([str(exe)], text=True).splitlines():
        cname, key, val = line.split()
        got[(cname, key)] = int(val)
    for cname, (cls, fields) in checks.items():
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for f in fields:
            assert got[(cname, f)] == getattr(cls, f).offset, (cname, f)
