"""Generate golden vectors by executing the reference's own attention source.

Run in the build container (it reads the reference checkout, which does not
exist where the GPU tests run):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

jax, flax and optax are not installable here, so the reference modules are
imported over a small numpy stand-in (``_NumpyJax`` / ``_MiniFlax`` below)
that provides only what the attention code touches: ``jax.numpy`` array
functions, ``jax.nn.softmax`` / ``sigmoid`` and flax ``Module`` /
``compact`` / ``param`` / ``Dense``. The reference functions then run
unmodified:

* confluence/confluence/model.py:201-264   build_attention_masks
* confluence/confluence/layers.py:113-174  GatedAttentionSublayer.__call__
* confluence/confluence/layers.py:42-110   QKNormedMultiHeadAttention.__call__

For each case the script records the inputs, the reference outputs and two
intermediates captured at module boundaries (the permuted hidden state and
permuted mask that reach the attention module, and the merged-head attention
output that reaches W_O). The stand-in's softmax restates jax's published
definition exp(x - max) / sum(exp(x - max)) (jax 0.9.0.1,
confluence/uv.lock:155-157).

Fixtures are written as compressed .npz next to this script.
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import rt_oracle as orc  # noqa: E402  (generator of synthetic inputs)


# ----------------------------------------------------------------------------
# numpy stand-in for jax / jax.numpy
# ----------------------------------------------------------------------------

class _AtSetter:
    def __init__(self, arr, idx):
        self.arr, self.idx = arr, idx

    def set(self, val):
        out = np.array(self.arr, copy=True)
        out[self.idx] = val
        return out.view(_JArray)


class _AtIndexer:
    def __init__(self, arr):
        self.arr = arr

    def __getitem__(self, idx):
        return _AtSetter(self.arr, idx)


class _JArray(np.ndarray):
    """ndarray with jax's functional ``.at[idx].set(v)`` update."""

    @property
    def at(self):
        return _AtIndexer(np.asarray(self))


def _make_jax(float_dtype):
    jnp = types.ModuleType("jax.numpy")
    jnp.int32 = np.int32
    jnp.bool_ = np.bool_
    jnp.float32 = float_dtype
    jnp.float16 = np.float16
    jnp.bfloat16 = float_dtype
    jnp.ndarray = np.ndarray
    jnp.arange = np.arange
    jnp.broadcast_to = np.broadcast_to
    jnp.eye = np.eye
    jnp.split = np.split
    jnp.maximum = np.maximum
    jnp.matmul = np.matmul
    jnp.sqrt = np.sqrt
    jnp.where = np.where
    jnp.take_along_axis = np.take_along_axis
    jnp.mean = np.mean
    jnp.array = np.array

    def zeros(shape, dtype=None):
        return np.zeros(shape, dtype=dtype).view(_JArray)

    def full(shape, fill, dtype=None):
        return np.full(shape, fill, dtype=dtype if dtype is not None else float_dtype)

    jnp.zeros = zeros
    jnp.full = full
    jnp.linalg = types.SimpleNamespace(norm=np.linalg.norm)

    def softmax(x, axis=-1):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / np.sum(e, axis=axis, keepdims=True)

    def sigmoid(x):
        return 1.0 / (1.0 + np.exp(-x))

    def silu(x):
        return x * sigmoid(x)

    jax = types.ModuleType("jax")
    jax.numpy = jnp
    jax.nn = types.SimpleNamespace(softmax=softmax, sigmoid=sigmoid, silu=silu)
    return jax, jnp


# ----------------------------------------------------------------------------
# minimal flax.linen stand-in
# ----------------------------------------------------------------------------

class _Scope:
    """Parameter tree + capture log shared by one reference invocation."""

    def __init__(self, params, rng, float_dtype):
        self.params = params
        self.stack = [params]
        self.rng = rng
        self.float_dtype = float_dtype
        self.captures = {}
        self.path = []


_ACTIVE: list[_Scope] = []


def _make_flax():
    linen = types.ModuleType("flax.linen")

    class Module:
        def __init_subclass__(cls, **kw):
            super().__init_subclass__(**kw)

        def __init__(self, *args, name=None, **kwargs):
            fields = [k for k in getattr(type(self), "__annotations__", {})]
            for k, v in zip(fields, args):
                setattr(self, k, v)
            for k, v in kwargs.items():
                setattr(self, k, v)
            self.name = name

        def param(self, pname, init_fn, shape):
            sc = _ACTIVE[-1]
            top = sc.stack[-1]
            if pname not in top:
                top[pname] = np.asarray(init_fn(sc.rng, shape), dtype=sc.float_dtype)
            return top[pname]

    def compact(fn):
        def wrapped(self, *args, **kwargs):
            sc = _ACTIVE[-1]
            pushed = False
            if self.name is not None:
                top = sc.stack[-1]
                sub = top.setdefault(self.name, {})
                sc.stack.append(sub)
                sc.path.append(self.name)
                pushed = True
            try:
                return fn(self, *args, **kwargs)
            finally:
                if pushed:
                    sc.stack.pop()
                    sc.path.pop()
        return wrapped

    def _lecun(rng, shape):
        return rng.standard_normal(shape) / np.sqrt(shape[0])

    def _xavier(rng, shape):
        lim = np.sqrt(6.0 / (shape[0] + shape[1]))
        return rng.uniform(-lim, lim, size=shape)

    class initializers:  # noqa: N801  (flax spelling)
        @staticmethod
        def zeros_init():
            return lambda rng, shape: np.zeros(shape)

        @staticmethod
        def xavier_uniform():
            return _xavier

    class Dense(Module):
        def __init__(self, features, use_bias=True, kernel_init=None, name=None):
            super().__init__(name=name)
            self.features = features
            self.use_bias = use_bias
            self.kernel_init = kernel_init or _lecun

        @compact
        def __call__(self, x):
            sc = _ACTIVE[-1]
            sc.captures["/".join(sc.path) + ":in"] = np.array(x, copy=True)
            kernel = self.param("kernel", self.kernel_init, (x.shape[-1], self.features))
            y = np.matmul(x, kernel)
            if self.use_bias:
                y = y + self.param("bias", initializers.zeros_init(), (self.features,))
            return y

    linen.Module = Module
    linen.compact = compact
    linen.Dense = Dense
    linen.initializers = initializers
    flax = types.ModuleType("flax")
    flax.linen = linen
    return flax, linen


def load_reference(reference_root, float_dtype=np.float32):
    """Import confluence.config / layers / model over the numpy stand-ins."""
    jax, jnp = _make_jax(float_dtype)
    flax, linen = _make_flax()
    saved = {k: sys.modules.get(k) for k in
             ("jax", "jax.numpy", "flax", "flax.linen", "confluence",
              "confluence.config", "confluence.layers", "confluence.model")}
    sys.modules.update({"jax": jax, "jax.numpy": jnp, "flax": flax, "flax.linen": linen})
    for k in ("confluence", "confluence.config", "confluence.layers", "confluence.model"):
        sys.modules.pop(k, None)
    sys.path.insert(0, os.path.join(reference_root, "confluence"))
    try:
        config = importlib.import_module("confluence.config")
        layers = importlib.import_module("confluence.layers")
        model = importlib.import_module("confluence.model")
    finally:
        sys.path.pop(0)
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return config, layers, model


def run_module(module, args, params, seed, float_dtype=np.float32):
    sc = _Scope(params, np.random.Generator(np.random.PCG64(seed)), float_dtype)
    _ACTIVE.append(sc)
    try:
        out = module(*args)
    finally:
        _ACTIVE.pop()
    return out, sc


# ----------------------------------------------------------------------------
# cases
# ----------------------------------------------------------------------------

def bookstore_batch():
    """The worked example of documentation/model_architecture/attention.md:42-75:
    rows 0..5 = order 1, customer 23, book 42, order 7, order 12, order 5;
    FK edges order1->{cust23, book42}, order7->cust23, order12->cust23,
    order5->book42. Each row gets two cells (orders: columns 0,1;
    customers: 2,3; books: 4,5), followed by 4 padding cells."""
    rows = [0, 1, 2, 3, 4, 5]
    table_cols = {0: (0, 1), 1: (2, 3), 2: (4, 5), 3: (0, 1), 4: (0, 1), 5: (0, 1)}
    seq_row_ids, column_ids = [], []
    for r in rows:
        for c in table_cols[r]:
            seq_row_ids.append(r)
            column_ids.append(c)
    s = len(seq_row_ids) + 4
    pad = [0] * len(seq_row_ids) + [1] * 4
    seq_row_ids += [0] * 4
    column_ids += [0] * 4
    fk = np.zeros((6, 6), dtype=np.uint8)
    for child, parent in [(0, 1), (0, 2), (3, 1), (4, 1), (5, 2)]:
        fk[child, parent] = 1
    return {
        "seq_row_ids": np.array([seq_row_ids], dtype=np.uint16),
        "column_ids": np.array([column_ids], dtype=np.int32),
        "is_padding": np.array([pad], dtype=np.uint8),
        "fk_adj": fk[None],
        "col_perm": np.arange(s, dtype=np.uint16)[None],
        "out_perm": np.arange(s, dtype=np.uint16)[None],
        "in_perm": np.arange(s, dtype=np.uint16)[None],
    }


MASK_CASES = {
    # name: generator arguments (seed, B, S, tables, cells_lo, cells_hi, p_fk, pad)
    "cfgA_s256": (11, 4, 256, 3, 4, 8, 0.6, 0.05),
    "ragged_s200": (12, 2, 200, 4, 2, 9, 0.8, 0.20),
    "dense_fk_s384": (13, 2, 384, 2, 3, 5, 1.0, 0.0),
    "no_fk_s128": (14, 1, 128, 5, 1, 12, 0.0, 0.5),
}

SUBLAYER_CASES = {
    # name: (mask seed args, H, Dh, kind)
    "cfgA_column": ((21, 1, 256, 3, 4, 8, 0.6, 0.05), 4, 32, orc.MASK_COLUMN),
    "cfgA_feature": ((22, 1, 256, 3, 4, 8, 0.6, 0.05), 4, 32, orc.MASK_FEATURE),
    "cfgA_neighbor": ((23, 1, 256, 3, 4, 8, 0.6, 0.05), 4, 32, orc.MASK_NEIGHBOR),
    "d64_feature_ragged": ((24, 1, 320, 4, 3, 10, 0.7, 0.1), 2, 64, orc.MASK_FEATURE),
}


def batch_to_ref(bt):
    return {k: np.asarray(v) for k, v in bt.items()}


def make_mask_fixture(model, bt):
    r = bt["fk_adj"].shape[1]
    outbound, inbound, column = model.build_attention_masks(batch_to_ref(bt), r)
    return {
        **{k: np.asarray(v) for k, v in bt.items()},
        "ref_outbound_bits": np.packbits(np.asarray(outbound, dtype=bool), axis=-1),
        "ref_inbound_bits": np.packbits(np.asarray(inbound, dtype=bool), axis=-1),
        "ref_column_bits": np.packbits(np.asarray(column, dtype=bool), axis=-1),
        "S": np.int64(bt["seq_row_ids"].shape[1]),
    }


def make_sublayer_fixture(config, layers, model, bt, h, dh, kind, seed):
    b, s = bt["seq_row_ids"].shape
    d = h * dh
    r = bt["fk_adj"].shape[1]
    outbound, inbound, column = model.build_attention_masks(batch_to_ref(bt), r)
    mask = {orc.MASK_COLUMN: column, orc.MASK_FEATURE: outbound,
            orc.MASK_NEIGHBOR: inbound}[kind]
    perm = {orc.MASK_COLUMN: bt["col_perm"], orc.MASK_FEATURE: bt["out_perm"],
            orc.MASK_NEIGHBOR: bt["in_perm"]}[kind]
    cfg = config.ModelConfig(d_model=d, n_heads=h, d_head=dh, max_seq_len=s, max_rows=r)
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((b, s, d)).astype(np.float32)
    params = {"sub": {
        "norm": {"gamma": (0.1 * rng.standard_normal(d)).astype(np.float32)},
        "mha": {"tau": (np.sqrt(dh) * (1.0 + 0.1 * rng.standard_normal((h, 1, 1))))
                .astype(np.float32)},
    }}
    sub = layers.GatedAttentionSublayer(config=cfg, output_scale=0.5, name="sub")

    # capture what reaches the attention module: the permuted state and mask
    orig_call = layers.QKNormedMultiHeadAttention.__call__
    seen = {}

    def spy(self, xx, mm):
        seen["x_perm"] = np.array(xx, copy=True)
        seen["mask_perm"] = np.array(mm, copy=True)
        return orig_call(self, xx, mm)

    layers.QKNormedMultiHeadAttention.__call__ = spy
    try:
        y, sc = run_module(sub, (x, mask, perm), params, seed + 1)
    finally:
        layers.QKNormedMultiHeadAttention.__call__ = orig_call
    p = sc.params["sub"]
    return {
        **{k: np.asarray(v) for k, v in bt.items()},
        "kind": np.int64(kind), "H": np.int64(h), "Dh": np.int64(dh),
        "x": x,
        "w_norm_gamma": np.asarray(p["norm"]["gamma"], dtype=np.float32),
        "w_qkv": np.asarray(p["mha"]["qkv"]["kernel"], dtype=np.float32),
        "tau": np.asarray(p["mha"]["tau"], dtype=np.float32).reshape(-1),
        "w_o": np.asarray(p["mha"]["wo"]["kernel"], dtype=np.float32),
        "w_gate": np.asarray(p["w_gate"]["kernel"], dtype=np.float32),
        "output_scale": np.float32(0.5),
        "ref_x_perm": seen["x_perm"].astype(np.float32),
        "ref_mask_perm_bits": np.packbits(seen["mask_perm"].astype(bool), axis=-1),
        "ref_attn_merged": sc.captures["sub/mha/wo:in"].astype(np.float32),
        "ref_y": np.asarray(y, dtype=np.float32),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference checkout (holds confluence/ and documentation/)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    config, layers, model = load_reference(args.reference)

    for name, gen in MASK_CASES.items():
        bt = orc.make_batch(*gen)
        np.savez_compressed(os.path.join(args.out, f"masks_{name}.npz"),
                            **make_mask_fixture(model, bt))
    np.savez_compressed(os.path.join(args.out, "masks_bookstore.npz"),
                        **make_mask_fixture(model, bookstore_batch()))

    for name, (gen, h, dh, kind) in SUBLAYER_CASES.items():
        bt = orc.make_batch(*gen)
        fx = make_sublayer_fixture(config, layers, model, bt, h, dh, kind, gen[0] * 7)
        np.savez_compressed(os.path.join(args.out, f"sublayer_{name}.npz"), **fx)
    print("wrote fixtures to", args.out)


if __name__ == "__main__":
    main()
