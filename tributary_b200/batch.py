"""Sampler-side batch layout: the cell orderings the kernels run under, and a
seeded synthetic batch generator with the shapes and distributions of the
benchmark configurations.

The reference builds its batches in Rust (headwater/src/sampler.rs); the
token metadata layout is headwater/src/python.rs:17-91 (seq_row_ids u16,
column_ids i32, is_padding u8, fk_adj[child][parent] u8, and the three
permutations col_perm / out_perm / in_perm as u16). The orderings here call
the library's host-side C ABI (rt_column_order, rt_rcm_order).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

MASK_COLUMN, MASK_FEATURE, MASK_NEIGHBOR, MASK_FULL = 0, 1, 2, 3
KIND_NAMES = ("column", "feature", "neighbor", "full")


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def column_order(column_ids: np.ndarray, is_padding: np.ndarray) -> np.ndarray:
    """[B,S] cells sorted by (padding last, column id, position) per sample
    (sampler.rs:655-668); returns uint16 [B,S]."""
    col = np.ascontiguousarray(column_ids, dtype=np.int32)
    pad = np.ascontiguousarray(is_padding, dtype=np.uint8)
    b, s = col.shape
    out = np.empty((b, s), dtype=np.uint16)
    _lib.check(_lib.load().rt_column_order(_ptr(col), _ptr(pad), b, s, _ptr(out)), "rt_column_order")
    return out


def rcm_order(fk_adj: np.ndarray, seq_row_ids: np.ndarray, is_padding: np.ndarray, outbound: bool) -> np.ndarray:
    """[B,S] reverse Cuthill-McKee cell order over each sample's FK graph
    (sampler.rs:672-784); outbound=True for the feature mask's order
    (out_perm), False for the neighbor mask's (in_perm)."""
    fk = np.ascontiguousarray(fk_adj, dtype=np.uint8)
    rows = np.ascontiguousarray(seq_row_ids, dtype=np.uint16)
    pad = np.ascontiguousarray(is_padding, dtype=np.uint8)
    b, s = rows.shape
    r = fk.shape[1]
    out = np.empty((b, s), dtype=np.uint16)
    _lib.check(_lib.load().rt_rcm_order(_ptr(fk), _ptr(rows), _ptr(pad), b, s, r, 1 if outbound else 0, _ptr(out)),
               "rt_rcm_order")
    return out


def make_batch(seed: int, B: int, S: int, n_tables: int, cells_lo: int, cells_hi: int, p_fk: float,
               pad_frac: float, parent_window: int | None = None, R: int | None = None,
               max_parents: int = 1) -> dict:
    """Seeded synthetic batch of cell-token metadata.

    Tables get fixed widths w_t ~ U[cells_lo, cells_hi] and global column ids
    base_t + 0..w_t-1 (column ids are global in the reference). Rows are
    emitted in order, each from a uniformly drawn table, with up to
    ``max_parents`` FK parents, each present with probability ``p_fk`` and
    drawn among the earlier rows (the latest ``parent_window`` when given):
    fk_adj[b, child, parent] = 1 (sampler.rs:516-526). Cells past
    S * (1 - pad_frac) are trailing padding (row 0, column 0). R defaults to the
    largest row count of the batch. Also returns col_perm / out_perm / in_perm.
    Draw order: widths, then per sample per row: table, then per parent slot
    the presence test and the parent index.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    widths = rng.integers(cells_lo, cells_hi + 1, size=n_tables)
    bases = np.concatenate([[0], np.cumsum(widths)[:-1]])
    n_valid = S - int(round(S * pad_frac))
    seq_row_ids = np.zeros((B, S), dtype=np.uint16)
    column_ids = np.zeros((B, S), dtype=np.int32)
    is_padding = np.ones((B, S), dtype=np.uint8)
    edges = []  # (sample, child, parent)
    rows_per_sample = []
    for b in range(B):
        pos, r = 0, 0
        while pos < n_valid:
            t = int(rng.integers(n_tables))
            for _ in range(max_parents):
                if r > 0 and rng.random() < p_fk:
                    lo = 0 if parent_window is None else max(0, r - parent_window)
                    edges.append((b, r, int(rng.integers(lo, r))))
            w = int(min(widths[t], n_valid - pos))
            column_ids[b, pos:pos + w] = bases[t] + np.arange(w)
            seq_row_ids[b, pos:pos + w] = r
            is_padding[b, pos:pos + w] = 0
            pos += w
            r += 1
        rows_per_sample.append(r)
    max_r = max([1] + rows_per_sample)
    R = max_r if R is None else R
    if R < max_r:
        raise ValueError(f"R={R} smaller than the {max_r} rows drawn")
    fk_adj = np.zeros((B, R, R), dtype=np.uint8)
    for b, child, parent in edges:
        fk_adj[b, child, parent] = 1
    return {
        "seq_row_ids": seq_row_ids,
        "column_ids": column_ids,
        "is_padding": is_padding,
        "fk_adj": fk_adj,
        "col_perm": column_order(column_ids, is_padding),
        "out_perm": rcm_order(fk_adj, seq_row_ids, is_padding, True),
        "in_perm": rcm_order(fk_adj, seq_row_ids, is_padding, False),
    }


def identity_order(B: int, S: int) -> np.ndarray:
    return np.broadcast_to(np.arange(S, dtype=np.uint16), (B, S)).copy()


def order_for_kind(batch: dict, kind: int) -> np.ndarray:
    """The ordering each mask kind runs under (confluence/confluence/layers.py:
    219-232 pairs outbound/feature with out_perm, inbound/neighbor with
    in_perm, column with col_perm); the full mask runs in token order."""
    b, s = batch["seq_row_ids"].shape
    return {MASK_COLUMN: batch["col_perm"], MASK_FEATURE: batch["out_perm"],
            MASK_NEIGHBOR: batch["in_perm"], MASK_FULL: identity_order(b, s)}[kind]


STYPE_IDENTIFIER, STYPE_NUMERICAL, STYPE_TIMESTAMP, STYPE_BOOLEAN, STYPE_CATEGORICAL, STYPE_TEXT, STYPE_IGNORED = range(7)


def make_cells(seed: int, B: int, S: int, n_tables: int, cells_lo: int, cells_hi: int, p_fk: float,
               pad_frac: float, max_parents: int = 1, d_text: int = 384, d_time: int = 8,
               n_categories: int = 4096, max_categories: int = 256, null_frac: float = 0.05,
               target_frac: float = 0.5, target_stype: int = STYPE_CATEGORICAL) -> dict:
    """A full training batch: the token metadata of make_batch plus seeded cell
    values by semantic type, in the layout the encoder consumes (the sampler
    fields of headwater/src/python.rs:17-91, with values drawn synthetically):
      stypes [B,S] int8 -- one semantic type per global column (padding:
        ignored); numeric_values [B,S] f32 ~ N(0,1) (z-scored);
      timestamp_values [B,S,d_time] f32 -- d_time-1 cyclic features sin/cos of
        uniform phases, then a z-scored scalar;
      bool_values [B,S] u8; categorical_ids [B,S] i32 into an n_categories row
        table, drawn from the first max_categories ids for the target column
        type; text_ids [B,S] i32 into text_vectors [U, d_text] ~ N(0,1)/sqrt(d_text);
      is_null [B,S] u8 (null_frac of real cells); is_target [B,S] u8 (target_frac
        of the cells of the target semantic type); target_stype; cat_start;
      col_table [C, d_text] and cat_table [n_categories, d_text] ~ N(0,1):
        the frozen column-name and category embeddings."""
    meta = make_batch(seed, B, S, n_tables, cells_lo, cells_hi, p_fk, pad_frac, max_parents=max_parents)
    rng = np.random.Generator(np.random.PCG64(seed + 0x5EED))
    real = meta["is_padding"] == 0
    n_cols = int(meta["column_ids"].max()) + 1
    col_stype = rng.choice(np.array([STYPE_NUMERICAL, STYPE_TIMESTAMP, STYPE_BOOLEAN, STYPE_CATEGORICAL,
                                     STYPE_TEXT, STYPE_IDENTIFIER], dtype=np.int8),
                           size=n_cols, p=[0.3, 0.15, 0.1, 0.3, 0.1, 0.05])
    col_stype[0] = target_stype  # at least one column of the target type
    stypes = np.where(real, col_stype[meta["column_ids"]], STYPE_IGNORED).astype(np.int8)
    phases = rng.uniform(0, 2 * np.pi, size=(B, S, (d_time - 1 + 1) // 2)).astype(np.float32)
    cyc = np.concatenate([np.sin(phases), np.cos(phases)], axis=-1)[..., :d_time - 1]
    ts = np.concatenate([cyc, rng.standard_normal((B, S, 1), dtype=np.float32)], axis=-1)
    n_text = max(1, B * S // 4)
    cat_ids = np.where(stypes == target_stype, rng.integers(0, max_categories, (B, S)),
                       rng.integers(0, n_categories, (B, S))).astype(np.int32)
    cells = dict(meta)
    cells.update(
        stypes=stypes,
        numeric_values=rng.standard_normal((B, S), dtype=np.float32),
        timestamp_values=np.ascontiguousarray(ts, dtype=np.float32),
        bool_values=rng.integers(0, 2, (B, S)).astype(np.uint8),
        categorical_ids=cat_ids,
        text_ids=rng.integers(0, n_text, (B, S)).astype(np.int32),
        text_vectors=(rng.standard_normal((n_text, d_text), dtype=np.float32) / np.sqrt(d_text)).astype(np.float32),
        is_null=((rng.random((B, S)) < null_frac) & real).astype(np.uint8),
        is_target=((rng.random((B, S)) < target_frac) & (stypes == target_stype)).astype(np.uint8),
        target_stype=int(target_stype),
        cat_start=0,
        col_table=rng.standard_normal((n_cols, d_text), dtype=np.float32),
        cat_table=rng.standard_normal((n_categories, d_text), dtype=np.float32),
    )
    return cells
