"""The MoE block's arithmetic restated in numpy (test infrastructure: the CUDA path's checker, never the product).

Each function names the reference code it restates (yibie/strata-mlx, paths within that project). Where the
reference's result depends on a rounding point (activations' type after SwiGLU, the combine's order) this
module rounds at the same point; products are otherwise taken in float64 so the oracle is the more exact side.
"""

import numpy as np

from .quants import dequantize

TOKENS_TILE = 16  # strata_mlx/blocks.py:581


def _as(dtype):
    return np.dtype(dtype).type


def matvec(blocks, kind, shape, x, idx, share=1):
    """out[p, r] = W[idx[p], r, :] . x[p // share]: `BlockSwitchLinear.__call__` (strata_mlx/blocks.py:538-554,
    kernel 196-220), float64 sums. x (pairs / share, cols); returns (pairs, rows) float64."""
    from .quants import row_bytes

    experts, rows, cols = shape
    idx = np.asarray(idx).reshape(-1).astype(np.int64)
    xs = np.asarray(x, dtype=np.float64).reshape(-1, cols)
    per_expert = rows * row_bytes(kind, cols)
    flat = np.asarray(blocks).reshape(-1)
    out = np.empty((idx.size, rows))
    for e in np.unique(idx):  # decode only the experts the pairs name
        w = dequantize(flat[e * per_expert : (e + 1) * per_expert], kind, (rows, cols)).astype(np.float64)
        sel = np.nonzero(idx == e)[0]
        out[sel] = xs[sel // share] @ w.T
    return out


def sigmoid_as(g, dtype):
    """`sigmoid` in float32 in MLX's two-branch form, rounded to `dtype` (strata_mlx/blocks.py:233-236)."""
    g32 = np.asarray(g, dtype=np.float32)
    with np.errstate(over="ignore"):
        y = np.float32(1) / (np.float32(1) + np.exp(np.abs(g32), dtype=np.float32))
    return np.where(g32 < 0, y, np.float32(1) - y).astype(dtype)


def swiglu(gate, up, dtype=np.float16):
    """mlx-lm's `swiglu(gate, up)` = silu(gate) * up in the activations' type: the sigmoid in float32 rounded to
    the type, then two products in the type (restated from strata_mlx/blocks.py:222-237)."""
    t = _as(dtype)
    g = np.asarray(gate).astype(dtype)
    u = np.asarray(up).astype(dtype)
    a = (g.astype(np.float32) * sigmoid_as(g, dtype).astype(np.float32)).astype(dtype)
    return (a.astype(np.float32) * u.astype(np.float32)).astype(t)


def router_logits(weight, x):
    """Router product: float16 weight (E, H) times x (T, H), float32 result (strata_mlx/fused.py:334-390)."""
    return (np.asarray(x, dtype=np.float64) @ np.asarray(weight, dtype=np.float64).T).astype(np.float32)


def top_k(logits, k):
    """Indices of the k largest of each row, largest first, ties to the lower index: what the reference's
    `_TOPK` kernel and `mx.argpartition(-logits, k-1)[..., :k]` give (strata_mlx/fused.py:395-436)."""
    logits = np.asarray(logits, dtype=np.float32)
    return np.argsort(-logits, axis=-1, kind="stable")[..., :k].astype(np.uint32)


def softmax_chosen(logits, idx):
    """`mx.softmax(take_along_axis(logits, idx), precise=True)` in float32 (strata_mlx/fused.py:491)."""
    chosen = np.take_along_axis(np.asarray(logits, dtype=np.float32), idx.astype(np.int64), axis=-1)
    e = np.exp(chosen - chosen.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def combine(y, w, g, s):
    """`moe_combine` (strata_mlx/fused.py:448-481): sum_k y_k w_k in float32 in MLX's col_reduce_small order
    (eight partial sums j = k mod 8, then the partials in order), rounded to the type; plus the shared expert
    times the type's sigmoid of its gate, each product rounded. y (T, K, D), w (T, K), g (T,), s (T, D)."""
    dt = y.dtype
    y32 = y.astype(np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    T, K, D = y.shape
    acc = np.zeros((T, D), dtype=np.float32)
    for j in range(min(8, K)):
        part = np.zeros((T, D), dtype=np.float32)
        for k in range(j, K, 8):
            part = (y32[:, k] * w32[:, k : k + 1]).astype(np.float32) + part
        acc = part if j == 0 else (part + acc).astype(np.float32)
    routed = acc.astype(dt)
    gate = (np.float32(1) / (np.float32(1) + np.exp(-np.asarray(g, dtype=np.float32)))).astype(dt)
    shared = (gate.astype(np.float32)[:, None] * s.astype(np.float32)).astype(dt)
    return (routed.astype(np.float32) + shared.astype(np.float32)).astype(dt)


def tiles_of(indices, experts):
    """The pairs of `indices` (..., k) in tiles of 16, each one expert's (strata_mlx/blocks.py:657-681).

    -> (tile_expert uint32 (most,), token uint32 (most*16,), where uint32 (pairs,)) with
    most = pairs // 16 + min(experts, pairs); a pair's position within its expert follows its flat index.
    """
    indices = np.asarray(indices)
    k = indices.shape[-1]
    flat = indices.reshape(-1).astype(np.int64)
    pairs = flat.size
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=experts)[:experts]
    tiles = (counts + TOKENS_TILE - 1) // TOKENS_TILE
    tile_end, pair_end = np.cumsum(tiles), np.cumsum(counts)
    expert = flat[order]
    slot = (tile_end - tiles)[expert] * TOKENS_TILE + np.arange(pairs) - (pair_end - counts)[expert]
    most = pairs // TOKENS_TILE + min(experts, pairs)
    token = np.zeros(most * TOKENS_TILE, dtype=np.uint32)
    token[slot] = order // k
    where = np.zeros(pairs, dtype=np.uint32)
    where[order] = slot
    tile_expert = (tile_end[None, :] <= np.arange(most)[:, None]).sum(axis=1)
    return tile_expert.astype(np.uint32), token, where


def tile_matmul(blocks, kind, shape, a, tile_expert):
    """out[p] = W[expert of p's tile] . a[p] with the weights rounded to a's type, float64 sums
    (strata_mlx/blocks.py:634-654). Rows of a tile that names no expert come back as NaN (undefined)."""
    experts, rows, cols = shape
    w = dequantize(blocks, kind, shape).astype(a.dtype).astype(np.float64)
    te = np.asarray(tile_expert).astype(np.int64)
    out = np.full((a.shape[0], rows), np.nan)
    for t, e in enumerate(te):
        if e < experts:
            out[16 * t : 16 * t + 16] = a[16 * t : 16 * t + 16].astype(np.float64) @ w[e].T
    return out


def switch_glu(x, idx, gate, up, down, dtype=np.float16):
    """down(swiglu(gate(x), up(x))) through each token's experts, pair at a time (strata_mlx/blocks.py:958-986,
    the BLOCK_GLU path): gate/up/down are (blocks, kind, shape). x (T, H); idx (T, k) -> (T, k, H) in dtype,
    gate/up outputs rounded to dtype as the reference's matvec returns them."""
    T, k = idx.shape
    g = matvec(*gate, x, idx, share=k).astype(dtype)
    u = matvec(*up, x, idx, share=k).astype(dtype)
    h = swiglu(g, u, dtype)
    y = matvec(*down, h, idx, share=1).astype(dtype)
    return y.reshape(T, k, -1)


def dense_mlp(x, gate, up, down, dtype=np.float16):
    """The shared expert: down(silu(gate(x)) * up(x)) with every product rounded to dtype (mlx-lm MLP,
    built at strata_mlx/load.py:419-421); gate/up/down are (blocks, kind, (rows, cols))."""
    T = x.shape[0]
    zeros = np.zeros(T, dtype=np.int64)
    g = matvec(gate[0], gate[1], (1, *gate[2]), x, zeros).astype(dtype)
    u = matvec(up[0], up[1], (1, *up[2]), x, zeros).astype(dtype)
    return matvec(down[0], down[1], (1, *down[2]), swiglu(g, u, dtype), zeros).astype(dtype)


def moe_block(x, router_w, k, experts, shared, shared_gate_w, dtype=np.float16, logits=None):
    """`_Routed.__call__` (strata_mlx/fused.py:487-497): router, top_k, softmax over the chosen, routed
    experts, shared expert and its sigmoid gate, combine. x (T, H) -> (T, H) dtype, plus (idx, w, logits).

    `logits` may be given (the device's own router product) so that a near-tie between the k-th and the
    (k+1)-th expert, which float32 sums in another order can flip, is decided the same way on both sides."""
    x = np.asarray(x).astype(dtype)
    if logits is None:
        logits = router_logits(router_w, x)
    idx = top_k(logits, k)
    w = softmax_chosen(logits, idx)
    y = switch_glu(x, idx, *experts, dtype=dtype)
    s = dense_mlp(x, *shared, dtype=dtype)
    g = (x.astype(np.float64) @ np.asarray(shared_gate_w, dtype=np.float64).reshape(-1)).astype(dtype)
    return combine(y, w, g, s), idx, w, logits


def partial_sums(y, w, lidx, experts, s):
    """One rank's float32 partials of an expert-parallel combine: sum over its pairs (lidx < experts) of y w in
    MLX's order, and its slice of the shared expert (float32). Returns (T, 2D) float32."""
    T, K, D = y.shape
    y32 = y.astype(np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    mask = (np.asarray(lidx).reshape(T, K) < experts)
    acc = np.zeros((T, D), dtype=np.float32)
    for j in range(min(8, K)):
        part = np.zeros((T, D), dtype=np.float32)
        for k in range(j, K, 8):
            term = (y32[:, k] * w32[:, k : k + 1]).astype(np.float32)
            part = np.where(mask[:, k : k + 1], term + part, part).astype(np.float32)
        acc = part if j == 0 else (part + acc).astype(np.float32)
    shared = np.zeros((T, D), dtype=np.float32) if s is None else s.astype(np.float32)
    return np.concatenate([acc, shared], axis=1)


def combine_sums(sums, g, dtype=np.float16):
    """The combine on summed partials: half(routed) + half(half(sigmoid(g)) half(shared)) (fused.py:448-462)."""
    D = sums.shape[1] // 2
    routed = sums[:, :D].astype(dtype)
    gate = (np.float32(1) / (np.float32(1) + np.exp(-np.asarray(g, dtype=np.float32)))).astype(dtype)
    shared = (gate.astype(np.float32)[:, None] * sums[:, D:].astype(dtype).astype(np.float32)).astype(dtype)
    return (routed.astype(np.float32) + shared.astype(np.float32)).astype(dtype)


def ep_reduce_combine(partials, g, dtype=np.float16):
    """The end of an expert-parallel decode step over the peer exchange: the ranks' float32 partials (each
    `partial_sums`' (T, 2D)) added in rank order, in float32, then `combine_sums`. No counterpart in the
    reference (one device); it is the combine of strata_mlx/fused.py:448-462 split across ranks."""
    total = np.asarray(partials[0], dtype=np.float32).copy()
    for p in partials[1:]:
        total = (total + np.asarray(p, dtype=np.float32)).astype(np.float32)
    return combine_sums(total, g, dtype)


def ep_plan(idx, experts, ranks):
    """The send side of a prompt chunk's expert-parallel exchange. No counterpart in the reference (one device);
    it splits `_Routed.__call__` (strata_mlx/fused.py:487-497) between top-k and `switch_mlp`: each pair goes to
    the rank owning its expert (idx // (experts / ranks)); destinations in rank order, one destination's pairs in
    pair order. Returns (counts[ranks] int32, where[pairs] int32 (-1: index out of range, not sent),
    send_expert[sent] uint32 (the expert in its owner's numbering), order[sent] (the pair of each place))."""
    flat = np.asarray(idx).reshape(-1).astype(np.int64)
    per = experts // ranks
    dest = np.where(flat < experts, flat // per, ranks)
    order = np.argsort(dest, kind="stable")
    order = order[dest[order] < ranks]
    counts = np.bincount(dest[dest < ranks], minlength=ranks).astype(np.int32)
    where = np.full(flat.size, -1, dtype=np.int32)
    where[order] = np.arange(order.size, dtype=np.int32)
    send_expert = (flat[order] - dest[order] * per).astype(np.uint32)
    return counts, where, send_expert, order


def combine_rows(y_rows, where, w, g, s):
    """`combine` with pair (t, j)'s expert output at y_rows[where[t k + j]] (0 for where -1)."""
    T, K = np.asarray(w).shape
    wh = np.asarray(where).reshape(T, K)
    yr = np.asarray(y_rows)
    if yr.shape[0] == 0:
        return combine(np.zeros((T, K, s.shape[-1]), dtype=yr.dtype), w, g, s)
    y = np.where((wh >= 0)[..., None], yr[np.maximum(wh, 0)], 0).astype(yr.dtype)
    return combine(y, w, g, s)
