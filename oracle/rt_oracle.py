"""CPU oracle for the Relational-Transformer masked attention path.

TEST INFRASTRUCTURE ONLY. This module is the checker: the tests, the smoke
check and the CPU-baseline leg of the benchmark import it. The product path
(the CUDA library under ``tributary_b200``) never calls it and has no CPU
fallback.

It restates, in numpy, the reference's arithmetic for the hot path:

* mask construction            confluence/confluence/model.py:201-264
* mask / token permutation     confluence/confluence/layers.py:139-167
* QK L2-norm and temperature   confluence/confluence/layers.py:63-80
* masked softmax attention     confluence/confluence/layers.py:82-97
  (third-party arithmetic: jax 0.9.0.1 ``jnp.matmul``, ``jnp.where``,
  ``jax.nn.softmax`` -- softmax(x) = exp(x - max x) / sum exp(x - max x))
* its backward                 (jax autodiff of the above under
                                ``jax.value_and_grad``, confluence/confluence/train.py:209)
* the sampler's permutations   headwater/src/sampler.rs:655-784
* the fk_adj layout            headwater/src/sampler.rs:516-526

Parity pin: the mask and forward restatements are checked against golden
vectors produced by executing the reference's own Python source
(``build_attention_masks``, ``GatedAttentionSublayer``,
``QKNormedMultiHeadAttention``) over a numpy stand-in for jax/flax; see
``tests/golden/make_golden.py``. The backward is pinned by central finite
differences of that same reference forward in float64. The sampler
permutations (Rust; no toolchain here) and the "full" mask kind (not in the
reference) are restatements without a reference run.

The tile vocabulary (128x128 tiles of the permuted mask, live / fully-live
bitmaps, compacted tile lists) is this build's own, defined in terms of the
permuted dense mask, and is what the prepass kernel must reproduce bit for
bit.
"""
from __future__ import annotations

from collections import deque

import numpy as np

TILE = 128

# Mask kinds. Reference names: outbound == RT "feature", inbound == RT
# "neighbor" (confluence/confluence/model.py:233-245).
MASK_COLUMN = 0
MASK_FEATURE = 1   # outbound: same row, or key row is an FK parent of the query row
MASK_NEIGHBOR = 2  # inbound: key row is an FK child of the query row
MASK_FULL = 3      # every non-padding pair (plus the diagonal)
MASK_NAMES = {MASK_COLUMN: "column", MASK_FEATURE: "feature",
              MASK_NEIGHBOR: "neighbor", MASK_FULL: "full"}


# ----------------------------------------------------------------------------
# Masks (confluence/confluence/model.py:201-264)
# ----------------------------------------------------------------------------

def build_attention_masks(seq_row_ids, fk_adj, column_ids, is_padding):
    """Dense [B,S,S] bool masks: (outbound, inbound, column, full).

    Follows confluence/confluence/model.py:211-262 step by step: gather
    fk_adj[b, r_i, r_j] (:227-230), outbound = same_row | fk_ij (:233-236),
    inbound = fk_adj[b, r_j, r_i] (:239-240), column = col_i == col_j
    (:243-245), AND with ~pad_i & ~pad_j (:248-254), OR the diagonal
    (:259-262). ``full`` = valid | diag is not in the reference; it is the
    fourth kind named by the benchmark configurations.
    """
    seq_row_ids = np.asarray(seq_row_ids).astype(np.int64)
    fk = np.asarray(fk_adj).astype(bool)
    pad = np.asarray(is_padding).astype(bool)
    col = np.asarray(column_ids)
    b, s = seq_row_ids.shape
    ri = seq_row_ids[:, :, None]
    rj = seq_row_ids[:, None, :]
    bidx = np.arange(b)[:, None, None]
    ri_b = np.broadcast_to(ri, (b, s, s))
    rj_b = np.broadcast_to(rj, (b, s, s))
    fk_ij = fk[bidx, ri_b, rj_b]
    fk_ji = fk[bidx, rj_b, ri_b]
    outbound = (ri == rj) | fk_ij
    inbound = fk_ji
    column = col[:, :, None] == col[:, None, :]
    valid = (~pad[:, :, None]) & (~pad[:, None, :])
    diag = np.eye(s, dtype=bool)[None]
    outbound = (outbound & valid) | diag
    inbound = (inbound & valid) | diag
    column = (column & valid) | diag
    full = valid | diag
    return outbound, inbound, column, full


def mask_for_kind(kind, seq_row_ids, fk_adj, column_ids, is_padding):
    outbound, inbound, column, full = build_attention_masks(
        seq_row_ids, fk_adj, column_ids, is_padding)
    return {MASK_COLUMN: column, MASK_FEATURE: outbound,
            MASK_NEIGHBOR: inbound, MASK_FULL: full}[kind]


def permute_mask(mask, perm):
    """mask_perm[b,i,j] = mask[b, perm[b,i], perm[b,j]]  (layers.py:144-152);
    indices past the end clamp to S-1, as jax gathers do."""
    perm = np.asarray(perm).astype(np.int64)
    b, s = perm.shape
    perm = np.minimum(perm, s - 1)
    bidx = np.arange(b)[:, None, None]
    return mask[bidx, perm[:, :, None], perm[:, None, :]]


def gather_tokens(x, perm):
    """x_perm[b,i,:] = x[b, perm[b,i], :]  (layers.py:139-142)."""
    perm = np.asarray(perm).astype(np.int64)
    return np.take_along_axis(x, perm[:, :, None], axis=1)


def scatter_tokens(x_perm, perm):
    """Inverse of gather_tokens via the inverse permutation (layers.py:159-167)."""
    perm = np.asarray(perm).astype(np.int64)
    b, s = perm.shape
    inv = np.zeros((b, s), dtype=np.int64)
    inv[np.arange(b)[:, None], perm] = np.arange(s)[None, :]
    return np.take_along_axis(x_perm, inv[:, :, None], axis=1)


# ----------------------------------------------------------------------------
# Attention core (confluence/confluence/layers.py:63-97)
# ----------------------------------------------------------------------------

def qk_normalize(q, k, tau):
    """q_hat = q / max(|q|, 1e-6) * tau_h ; k_hat = k / max(|k|, 1e-6).

    layers.py:65-80; q, k are [B,H,S,Dh], tau is [H] (the reference keeps it
    as an [H,1,1] parameter initialised to sqrt(Dh)).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    qn = q / np.maximum(np.linalg.norm(q, axis=-1, keepdims=True), np.float32(1e-6))
    kn = k / np.maximum(np.linalg.norm(k, axis=-1, keepdims=True), np.float32(1e-6))
    tau = np.asarray(tau, dtype=np.float32).reshape(1, -1, 1, 1)
    return (qn * tau).astype(np.float32), kn.astype(np.float32)


def attention_fwd(q, k, v, mask, scale, dtype=np.float32):
    """Masked softmax attention; returns (o, lse).

    s = q k^T * scale (layers.py:83, scale = 1/sqrt(Dh)); s = where(mask, s,
    -1e9) (:86-88); p = softmax(s) (:90); o = p v (:93-94). ``mask`` is
    [B,S,S] (broadcast over heads, :85-86). lse = logsumexp of the filled
    logits (natural log); every row holds its diagonal, so the -1e9 entries
    contribute exactly zero in float32 and lse equals the log-sum over live
    keys.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * dtype(scale)
    s = np.where(mask[:, None], s, dtype(-1e9))
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(axis=-1, keepdims=True)
    p = e / l
    o = np.matmul(p, v)
    lse = (m + np.log(l))[..., 0]
    return o.astype(dtype), lse.astype(dtype)


def attention_bwd(q, k, v, o, do, mask, scale, dtype=np.float32):
    """Analytic gradients (dq, dk, dv) of attention_fwd.

    The reference has no hand-written backward; jax autodiff differentiates
    layers.py:83-94. With p = softmax(s): dv = p^T do; dp = do v^T;
    ds = p * (dp - rowsum(do * o)); dq = scale * ds k; dk = scale * ds^T q.
    Masked entries have p = 0 and so receive no gradient, as in autodiff of
    ``jnp.where``.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    o = np.asarray(o, dtype=dtype)
    do = np.asarray(do, dtype=dtype)
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * dtype(scale)
    s = np.where(mask[:, None], s, dtype(-1e9))
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    p = e / e.sum(axis=-1, keepdims=True)
    dv = np.matmul(np.swapaxes(p, -1, -2), do)
    dp = np.matmul(do, np.swapaxes(v, -1, -2))
    delta = (do * o).sum(axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = np.matmul(ds, k) * dtype(scale)
    dk = np.matmul(np.swapaxes(ds, -1, -2), q) * dtype(scale)
    return dq.astype(dtype), dk.astype(dtype), dv.astype(dtype)


# ----------------------------------------------------------------------------
# Tile occupancy (the prepass contract)
# ----------------------------------------------------------------------------

def n_tiles(s):
    return (s + TILE - 1) // TILE


def padded_tile_mask(mask_perm):
    """[B,S,S] -> [B,T*128,T*128] with out-of-range rows/cols false."""
    b, s, _ = mask_perm.shape
    t = n_tiles(s)
    out = np.zeros((b, t * TILE, t * TILE), dtype=bool)
    out[:, :s, :s] = mask_perm
    return out


def tile_occupancy(mask_perm):
    """Per-(b, q-tile, k-tile) live / fully-live flags, shape [B,T,T] bool.

    A tile is live iff any in-range element is true. It is fully live iff it
    is entirely in range (no ragged edge) and every element is true.
    """
    b, s, _ = mask_perm.shape
    t = n_tiles(s)
    m = padded_tile_mask(mask_perm).reshape(b, t, TILE, t, TILE)
    live = m.any(axis=(2, 4))
    full = m.all(axis=(2, 4))
    return live, full


def pack_bits_rows(flags):
    """[..., N] bool -> [..., ceil(N/32)] uint32, bit j%32 of word j//32 = flag j."""
    flags = np.asarray(flags, dtype=bool)
    n = flags.shape[-1]
    w = (n + 31) // 32
    padded = np.zeros(flags.shape[:-1] + (w * 32,), dtype=np.uint64)
    padded[..., :n] = flags
    padded = padded.reshape(flags.shape[:-1] + (w, 32))
    weights = (np.uint64(1) << np.arange(32, dtype=np.uint64))
    return (padded * weights).sum(axis=-1).astype(np.uint32)


def tile_bitmaps(mask_perm):
    """(live_bits, full_bits), each [B,T,ceil(T/32)] uint32."""
    live, full = tile_occupancy(mask_perm)
    return pack_bits_rows(live), pack_bits_rows(full)


def tile_lists(mask_perm):
    """Compacted tile lists in both orders, ascending.

    q2k: for each (b, qt) in row-major order, the live kt; k2q: for each
    (b, kt), the live qt. Entries carry the fully-live flag in bit 31.
    Returns (q2k_ptr, q2k_idx, k2q_ptr, k2q_idx) as int32 arrays.
    """
    live, full = tile_occupancy(mask_perm)
    b, t, _ = live.shape
    flag = np.int64(1) << 31

    def build(lv, fl):
        ptr = [0]
        idx = []
        for bb in range(b):
            for r in range(t):
                cols = np.nonzero(lv[bb, r])[0]
                for c in cols:
                    idx.append(int(c) | (int(flag) if fl[bb, r, c] else 0))
                ptr.append(len(idx))
        idx = np.array(idx, dtype=np.int64)
        idx = np.where(idx >= flag, idx - (1 << 32), idx)  # two's complement int32
        return np.array(ptr, dtype=np.int32), idx.astype(np.int32)

    q2k_ptr, q2k_idx = build(live, full)
    k2q_ptr, k2q_idx = build(np.swapaxes(live, 1, 2), np.swapaxes(full, 1, 2))
    return q2k_ptr, q2k_idx, k2q_ptr, k2q_idx


def tile_mask_words(mask_perm):
    """Per-tile element bits, [B,T,T,128,4] uint32 (query-major).

    Word w of row i in tile (qt, kt) holds keys kt*128 + 32w .. +31 of query
    qt*128 + i, bit j%32 = key j. Out-of-range rows and keys are zero.
    """
    b, s, _ = mask_perm.shape
    t = n_tiles(s)
    m = padded_tile_mask(mask_perm).reshape(b, t, TILE, t, TILE).transpose(0, 1, 3, 2, 4)
    return pack_bits_rows(m)  # [B, T(q), T(k), 128(i), 4]


def tile_mask_words_t(mask_perm):
    """Key-major twin of tile_mask_words: [B,T(k),T(q),128(key),4] over queries."""
    return tile_mask_words(np.swapaxes(mask_perm, 1, 2))


def live_fraction(mask_perm):
    live, _ = tile_occupancy(mask_perm)
    return float(live.mean())


# ----------------------------------------------------------------------------
# Sampler permutations (headwater/src/sampler.rs:655-784)
# ----------------------------------------------------------------------------

def compute_col_perm(column_ids, is_padding):
    """Stable argsort by (is_padding, column_id, position); sampler.rs:655-668."""
    column_ids = np.asarray(column_ids)
    is_padding = np.asarray(is_padding)
    s = column_ids.shape[0]
    pos = np.arange(s)
    order = np.lexsort((pos, column_ids.astype(np.int64), is_padding.astype(np.int64)))
    return order.astype(np.uint16)


def compute_rcm_perm(fk_adj, seq_row_ids, is_padding, outbound):
    """Reverse Cuthill-McKee row order, then cells sorted by (pad, rank, pos).

    Restates sampler.rs:672-784 exactly, including its tie-breaking: the BFS
    start is the first unvisited *used* row of minimum out-degree (Rust
    ``min_by_key`` keeps the first minimum), else the first unvisited row;
    neighbours are visited in a stable sort by degree; the order is reversed.
    ``outbound`` uses adjacency (I + fk_adj) with self loops dropped, the
    inbound variant uses fk_adj^T.
    """
    fk = np.asarray(fk_adj).astype(bool)
    r = fk.shape[0]
    seq_row_ids = np.asarray(seq_row_ids).astype(np.int64)
    is_padding = np.asarray(is_padding)
    s = seq_row_ids.shape[0]
    a = fk if outbound else fk.T
    adj = []
    for i in range(r):
        row = a[i].copy()
        row[i] = False
        adj.append([int(j) for j in np.nonzero(row)[0]])
    deg = [len(x) for x in adj]
    used = np.zeros(r, dtype=bool)
    for pos in range(s):
        if is_padding[pos] == 0 and seq_row_ids[pos] < r:
            used[seq_row_ids[pos]] = True
    visited = np.zeros(r, dtype=bool)
    order = []
    while len(order) < r:
        start = None
        best = None
        for i in range(r):
            if not visited[i] and used[i] and (best is None or deg[i] < best):
                best = deg[i]
                start = i
        if start is None:
            for i in range(r):
                if not visited[i]:
                    start = i
                    break
        if start is None:
            break
        queue = deque([start])
        visited[start] = True
        while queue:
            node = queue.popleft()
            order.append(node)
            nb = [n for n in adj[node] if not visited[n]]
            nb.sort(key=lambda n: deg[n])  # stable, like sort_by_key
            for n in nb:
                if not visited[n]:
                    visited[n] = True
                    queue.append(n)
    order.reverse()
    for i in range(r):
        if not visited[i]:
            order.append(i)
    rank = np.zeros(r, dtype=np.int64)
    for k, row in enumerate(order):
        rank[row] = k
    big = np.iinfo(np.int64).max
    cell_rank = np.array([rank[x] if x < r else big for x in seq_row_ids], dtype=np.int64)
    pos = np.arange(s)
    perm = np.lexsort((pos, cell_rank, is_padding.astype(np.int64)))
    return perm.astype(np.uint16)


# ----------------------------------------------------------------------------
# Synthetic batch generator (shapes and distributions of the benchmark configs)
# ----------------------------------------------------------------------------

def make_batch(seed, B, S, n_tables, cells_lo, cells_hi, p_fk, pad_frac,
               parent_window=None, R=None, max_parents=1):
    """Seeded synthetic sampler batch in the headwater layout.

    Each table t has a fixed width w_t ~ U[cells_lo, cells_hi] and global
    column ids base_t + 0..w_t-1 (column ids are global in the reference,
    documentation/model_architecture/batch_structure.md:46-47). Rows are
    emitted in order with a uniformly drawn table; a row draws up to
    ``max_parents`` FK parents, each present with probability p_fk, among the
    earlier rows of the sample (the most recent ``parent_window`` rows when
    given, else all of them), recorded as fk_adj[b, child, parent] = 1
    (sampler.rs:516-526; a row may have several FK parents). Cells past
    S*(1-pad_frac) are trailing padding (seq_row_id 0, column id 0, as the
    sampler leaves them, sampler.rs:336-347). R defaults to the largest row
    count in the batch.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    widths = rng.integers(cells_lo, cells_hi + 1, size=n_tables)
    bases = np.concatenate([[0], np.cumsum(widths)[:-1]])
    n_valid = S - int(round(S * pad_frac))
    seq_row_ids = np.zeros((B, S), dtype=np.uint16)
    column_ids = np.zeros((B, S), dtype=np.int32)
    is_padding = np.ones((B, S), dtype=np.uint8)
    parents = []
    for b in range(B):
        pos = 0
        par = []
        while pos < n_valid:
            t = int(rng.integers(n_tables))
            r = len(par)
            ps = []
            for _ in range(max_parents):
                if r > 0 and rng.random() < p_fk:
                    lo = 0 if parent_window is None else max(0, r - parent_window)
                    ps.append(int(rng.integers(lo, r)))
            w = int(min(widths[t], n_valid - pos))
            column_ids[b, pos:pos + w] = bases[t] + np.arange(w)
            seq_row_ids[b, pos:pos + w] = r
            is_padding[b, pos:pos + w] = 0
            par.append(ps)
            pos += w
        parents.append(par)
    max_r = max(1, max(len(p) for p in parents))
    if R is None:
        R = max_r
    if R < max_r:
        raise ValueError(f"R={R} smaller than the {max_r} rows drawn")
    fk_adj = np.zeros((B, R, R), dtype=np.uint8)
    for b, par in enumerate(parents):
        for child, ps in enumerate(par):
            for parent in ps:
                fk_adj[b, child, parent] = 1
    col_perm = np.stack([compute_col_perm(column_ids[b], is_padding[b]) for b in range(B)])
    out_perm = np.stack([compute_rcm_perm(fk_adj[b], seq_row_ids[b], is_padding[b], True)
                         for b in range(B)])
    in_perm = np.stack([compute_rcm_perm(fk_adj[b], seq_row_ids[b], is_padding[b], False)
                        for b in range(B)])
    return {
        "seq_row_ids": seq_row_ids,
        "column_ids": column_ids,
        "is_padding": is_padding,
        "fk_adj": fk_adj,
        "col_perm": col_perm,
        "out_perm": out_perm,
        "in_perm": in_perm,
    }


def identity_perm(B, S):
    return np.broadcast_to(np.arange(S, dtype=np.uint16), (B, S)).copy()


def perm_for_kind(batch, kind):
    """The permutation each kind runs under: col_perm for column, out_perm for
    feature (outbound), in_perm for neighbor (inbound) -- the pairing of
    confluence/confluence/layers.py:219-232 -- and the identity for full."""
    b, s = batch["seq_row_ids"].shape
    return {MASK_COLUMN: batch["col_perm"], MASK_FEATURE: batch["out_perm"],
            MASK_NEIGHBOR: batch["in_perm"], MASK_FULL: identity_perm(b, s)}[kind]


def make_qkv(seed, B, H, S, Dh, dtype=np.float32):
    """q_hat, k_hat, v, d_out: N(0,1) draws, q and k L2-normalised with tau =
    sqrt(Dh) folded into q (layers.py:70-80)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    q = rng.standard_normal((B, H, S, Dh), dtype=np.float32)
    k = rng.standard_normal((B, H, S, Dh), dtype=np.float32)
    v = rng.standard_normal((B, H, S, Dh), dtype=np.float32)
    do = rng.standard_normal((B, H, S, Dh), dtype=np.float32)
    qh, kh = qk_normalize(q, k, np.full(H, np.sqrt(Dh), dtype=np.float32))
    return qh.astype(dtype), kh.astype(dtype), v.astype(dtype), do.astype(dtype)


# ----------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as the device's cvt.rn.bf16.f32)
# ----------------------------------------------------------------------------

def to_bf16_bits(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    out[nan] = 0x7FC0
    return out


def from_bf16_bits(b):
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x):
    return from_bf16_bits(to_bf16_bits(x))
