"""Generates tests/golden/composed_small.npz.

The reference's Python layer functions (python/oxitorch/nn/functional.py of
SirBlocky7747/oxitorch) are executed *unmodified* from the reference checkout,
with their ``_native`` module replaced by the oracle's restatement of the Rust
``Tensor``/``Var`` engine (oracle/oxiref.py).  The outputs and gradients of
each F.* call on small seeded inputs are stored together with the inputs.

The committed fixtures pin two things at once: the oracle's restated F.*
compositions must reproduce them bit for bit (tests/test_golden.py), and the
CUDA kernels are checked against them on the GPU.  The reference checkout is
only needed to regenerate the file:

    python tests/golden/make_golden.py /path/to/oxitorch
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oxiref as R  # noqa: E402


def load_reference_functional(ref_root):
    """Imports <ref_root>/python/oxitorch/nn/functional.py with oxitorch._native
    bound to the oracle."""
    native = types.ModuleType("oxitorch._native")
    native.from_numpy = R.from_numpy
    pkg = types.ModuleType("oxitorch")
    pkg.__path__ = []
    pkg._native = native
    nn = types.ModuleType("oxitorch.nn")
    nn.__path__ = []
    sys.modules.update({"oxitorch": pkg, "oxitorch._native": native, "oxitorch.nn": nn})
    path = os.path.join(ref_root, "python", "oxitorch", "nn", "functional.py")
    spec = importlib.util.spec_from_file_location("oxitorch.nn.functional", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cases():
    """(name, builder) pairs; each builder takes an F module and returns a dict
    of float32 arrays (inputs first, then outputs/grads)."""
    out = []

    def rms(F, seed, m, n):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((m, n), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        dy = rng.standard_normal((m, n), dtype=np.float32)
        xt, wt = R.from_numpy(x, True), R.from_numpy(w, True)
        y = F.rms_norm(xt, wt, 1e-6)
        y.backward(R.from_numpy(dy))
        return dict(x=x, w=w, dy=dy, y=y.numpy(), dx=xt.grad.numpy(), dw=wt.grad.numpy())

    def ln_gelu(F, seed, m, n):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((m, n), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        dy = rng.standard_normal((m, n), dtype=np.float32)
        xt, wt, bt = R.from_numpy(x, True), R.from_numpy(w, True), R.from_numpy(b, True)
        y = F.gelu(F.layer_norm(xt, wt, bt, 1e-5))
        y.backward(R.from_numpy(dy))
        return dict(x=x, w=w, b=b, dy=dy, y=y.numpy(), dx=xt.grad.numpy(), dw=wt.grad.numpy(),
                    db=bt.grad.numpy())

    def ln(F, seed, m, n):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((m, n), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        dy = rng.standard_normal((m, n), dtype=np.float32)
        xt, wt, bt = R.from_numpy(x, True), R.from_numpy(w, True), R.from_numpy(b, True)
        y = F.layer_norm(xt, wt, bt, 1e-5)
        y.backward(R.from_numpy(dy))
        return dict(x=x, w=w, b=b, dy=dy, y=y.numpy(), dx=xt.grad.numpy(), dw=wt.grad.numpy(),
                    db=bt.grad.numpy())

    def softmax(F, seed, m, n, log):
        rng = np.random.default_rng(seed)
        x = (rng.standard_normal((m, n), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
        x[rng.random((m, n)) < 0.01] = 20.0
        dy = rng.standard_normal((m, n), dtype=np.float32)
        xt = R.from_numpy(x, True)
        y = (F.log_softmax if log else F.softmax)(xt, -1)
        y.backward(R.from_numpy(dy))
        return dict(x=x, dy=dy, y=y.numpy(), dx=xt.grad.numpy())

    def ce(F, seed, m, n):
        rng = np.random.default_rng(seed)
        x = (rng.standard_normal((m, n), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
        x[rng.random((m, n)) < 0.01] = 20.0
        t = rng.integers(0, n, m)
        xt = R.from_numpy(x, True)
        loss = F.cross_entropy(xt, [int(v) for v in t])
        loss.backward()
        return dict(x=x, targets=t.astype(np.int64), loss=np.array(loss.item(), np.float32),
                    dx=xt.grad.numpy())

    def silu(F, seed, m, n):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((m, n), dtype=np.float32)
        dy = rng.standard_normal((m, n), dtype=np.float32)
        xt = R.from_numpy(x, True)
        y = F.silu(xt)
        y.backward(R.from_numpy(dy))
        return dict(x=x, dy=dy, y=y.numpy(), dx=xt.grad.numpy())

    def swiglu(F, seed, m, n):
        rng = np.random.default_rng(seed)
        g = rng.standard_normal((m, n), dtype=np.float32)
        u = rng.standard_normal((m, n), dtype=np.float32)
        dh = rng.standard_normal((m, n), dtype=np.float32)
        gt, ut = R.from_numpy(g, True), R.from_numpy(u, True)
        h = F.silu(gt) * ut
        h.backward(R.from_numpy(dh))
        return dict(g=g, u=u, dh=dh, h=h.numpy(), dg=gt.grad.numpy(), du=ut.grad.numpy())

    def emb(F, seed, v, d, n):
        rng = np.random.default_rng(seed)
        table = rng.standard_normal((v, d), dtype=np.float32)
        ids = np.minimum(rng.zipf(1.1, n) - 1, v - 1).astype(np.int64)
        dout = rng.standard_normal((n, d), dtype=np.float32)
        tt = R.from_numpy(table, True)
        out = F.embedding([int(i) for i in ids], tt)
        out.backward(R.from_numpy(dout))
        return dict(table=table, ids=ids, dout=dout, out=out.numpy(), dtable=tt.grad.numpy())

    out += [("rms_4x4096", lambda F: rms(F, 101, 4, 4096)),
            ("rms_7x1001", lambda F: rms(F, 102, 7, 1001)),
            ("rms_3x4", lambda F: rms(F, 103, 3, 4))]
    out += [("lngelu_4x4096", lambda F: ln_gelu(F, 201, 4, 4096)),
            ("lngelu_5x777", lambda F: ln_gelu(F, 202, 5, 777)),
            ("ln_6x512", lambda F: ln(F, 203, 6, 512))]
    out += [("softmax_4x3000", lambda F: softmax(F, 301, 4, 3000, False)),
            ("logsoftmax_4x3000", lambda F: softmax(F, 302, 4, 3000, True)),
            ("logsoftmax_3x5", lambda F: softmax(F, 303, 3, 5, True))]
    out += [("ce_8x3200", lambda F: ce(F, 304, 8, 3200)),
            ("ce_5x7", lambda F: ce(F, 305, 5, 7))]
    out += [("silu_4x1000", lambda F: silu(F, 501, 4, 1000)),
            ("swiglu_4x1100", lambda F: swiglu(F, 502, 4, 1100))]
    out += [("emb_300x32_n1500", lambda F: emb(F, 401, 300, 32, 1500)),
            ("emb_40x6_n50", lambda F: emb(F, 402, 40, 6, 50))]
    return out


def main(ref_root):
    ref_F = load_reference_functional(ref_root)
    blobs = {}
    for name, build in cases():
        got_ref = build(ref_F)
        got_mine = build(R)  # the oracle's restated compositions
        for k, v in got_ref.items():
            if not np.array_equal(v, got_mine[k], equal_nan=True):
                raise SystemExit(f"{name}.{k}: restated F.* differs from the reference's functional.py")
            blobs[f"{name}.{k}"] = v
        print(f"{name}: ok ({', '.join(got_ref)})")
    path = os.path.join(HERE, "composed_small.npz")
    np.savez_compressed(path, **blobs)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
