"""The C ABI used from plain C (tests/c_abi/abi_roundtrip.c: the CUDA runtime
for memory and copies, include/rt_attention.h for the rest; no Python, no
PyTorch): the tile plan, the forward and the backward of one problem, checked
against the oracle."""
import os
import subprocess

import numpy as np
import pytest

from oracle import rt_oracle as orc
from rt_cases import TOL_LSE, TOL_OUT, max_rel

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _build(tmp):
    exe = os.path.join(tmp, "abi_roundtrip")
    lib_dir = os.path.join(REPO, "tributary_b200")
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-I", os.path.join(REPO, "include"), "-I", "/usr/local/cuda/include",
           os.path.join(REPO, "tests", "c_abi", "abi_roundtrip.c"), "-L", lib_dir, "-l:libtributary_b200.so",
           "-L", "/usr/local/cuda/lib64", "-lcudart", "-lm", f"-Wl,-rpath,{lib_dir}", "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True)
    return exe


@pytest.mark.parametrize("kind,dh", [(1, 64), (0, 32)])
def test_plain_c_caller_matches_oracle(cuda_lib, tmp_path, kind, dh):
    exe = _build(str(tmp_path))
    bt = orc.make_batch(111, 2, 1000, 6, 4, 16, 0.7, 0.1, None, None, 2)
    b, s = bt["seq_row_ids"].shape
    r = bt["fk_adj"].shape[1]
    h = 3
    perm = orc.perm_for_kind(bt, kind)
    q, k, v, do = (orc.round_bf16(x) for x in orc.make_qkv(112 + kind, b, h, s, dh))
    files = {"perm.u16": perm.astype(np.uint16), "rows.u16": bt["seq_row_ids"].astype(np.uint16),
             "cols.i32": bt["column_ids"].astype(np.int32), "pad.u8": bt["is_padding"].astype(np.uint8),
             "fk.u8": bt["fk_adj"].astype(np.uint8), "q.bf16": orc.to_bf16_bits(q), "k.bf16": orc.to_bf16_bits(k),
             "v.bf16": orc.to_bf16_bits(v), "do.bf16": orc.to_bf16_bits(do)}
    for name, arr in files.items():
        np.ascontiguousarray(arr).tofile(os.path.join(tmp_path, name))
    proc = subprocess.run([exe, str(tmp_path), str(b), str(s), str(r), str(h), str(dh), str(kind)],
                          capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr

    def load(name, dtype):
        return np.fromfile(os.path.join(tmp_path, name), dtype=dtype)

    mask = orc.permute_mask(orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"], bt["column_ids"],
                                              bt["is_padding"]), perm)
    live, _ = orc.tile_occupancy(mask)
    assert int(load("nnz.i32", np.int32)[0]) == int(live.sum())
    scale = 1.0 / np.sqrt(dh)
    o_ref, lse_ref = orc.attention_fwd(q, k, v, mask, scale, dtype=np.float64)
    grads_ref = orc.attention_bwd(q, k, v, o_ref, do, mask, scale, dtype=np.float64)
    shape = (b, h, s, dh)
    o = orc.from_bf16_bits(load("o.bf16", np.uint16)).reshape(shape)
    assert max_rel(o, o_ref) < TOL_OUT
    np.testing.assert_allclose(load("lse.f32", np.float32).reshape(b, h, s), lse_ref, atol=TOL_LSE, rtol=0)
    for name, ref in zip(("dq", "dk", "dv"), grads_ref):
        got = orc.from_bf16_bits(load(f"{name}.bf16", np.uint16)).reshape(shape)
        assert max_rel(got, ref) < TOL_OUT, name
