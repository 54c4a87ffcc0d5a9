"""Torch-facing wrappers of the native ops.

Every op: checks that inputs are CUDA float32 tensors, makes them contiguous,
allocates outputs and workspace through torch's caching allocator, and enqueues
the kernels on the current CUDA stream.  There is no CPU path: on a machine
without a GPU the ops raise ``CUDANotAvailableError`` (the reference's error,
flash_eq/cuda/block_diagonal.py:34-55).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class CUDANotAvailableError(RuntimeError):
    """Raised when CUDA is required but not available (flash_eq/cuda/block_diagonal.py:34-36)."""


def _require_cuda(*tensors):
    if not torch.cuda.is_available():
        raise CUDANotAvailableError(
            "flash-eq requires a CUDA-capable GPU. No CUDA device was detected."
        )
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("flash-eq ops need CUDA tensors; got a tensor on " + str(t.device))
    return _lib.load()


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.float32:
        raise TypeError(f"{name}: flash-eq B200 kernels compute in float32; got {t.dtype}")
    return t.contiguous()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


EDGEWISE_WS_CAP = None     # scratch cap of one edgewise call in bytes; None: 1/8 of the device memory, >= 1 GiB


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def dim_of(lvals) -> int:
    return sum(2 * int(l) + 1 for l in lvals)


# ---------------------------------------------------------------------------
def wigner_basis(directions: torch.Tensor, lvals, layout: int = _lib.FEQ_BASIS_MFIRST) -> torch.Tensor:
    lib = _require_cuda(directions)
    directions = _f32(directions, "directions")
    if directions.dim() != 2 or directions.shape[-1] != 3:
        raise ValueError(f"directions must be (E, 3); got {tuple(directions.shape)}")
    E = directions.shape[0]
    d = dim_of(lvals)
    out = torch.empty(E, d, d, device=directions.device, dtype=torch.float32)
    arr, n = _lib.i32_array(lvals)
    rc = lib.feq_wigner_basis(_p(directions), E, arr, n, layout, _p(out), _stream(directions.device))
    _lib.check(rc, "feq_wigner_basis")
    return out


def edge_binning(distances: torch.Tensor, p1: float, p2: float, num_bins: int, log_bins: bool):
    lib = _require_cuda(distances)
    distances = _f32(distances, "distances")
    E = distances.numel()
    lo = torch.empty(E, dtype=torch.int32, device=distances.device)
    t = torch.empty(E, dtype=torch.float32, device=distances.device)
    rc = lib.feq_edge_binning(_p(distances), E, float(p1), float(p2), int(num_bins), int(bool(log_bins)),
                              _p(lo), _p(t), _stream(distances.device))
    _lib.check(rc, "feq_edge_binning")
    return lo, t


def edge_sort(keys: torch.Tensor, num_keys: int):
    """Stable sort of edge ids by key -> (perm int64 (E,), offsets int64 (num_keys+1,), status int32 (1,))."""
    lib = _require_cuda(keys)
    keys = keys.contiguous()
    E = keys.numel()
    dev = keys.device
    perm = torch.empty(E, dtype=torch.int64, device=dev)
    offsets = torch.empty(num_keys + 1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.feq_edge_sort_workspace_bytes(E, num_keys)
    ws = _workspace(ws_bytes, dev)
    if keys.dtype == torch.int64:
        fn = lib.feq_edge_sort_i64
    elif keys.dtype == torch.int32:
        fn = lib.feq_edge_sort
    else:
        raise TypeError("edge_sort keys must be int32 or int64")
    rc = fn(_p(keys), E, int(num_keys), _p(perm), _p(offsets), _p(status), _p(ws), ws.numel(), _stream(dev))
    _lib.check(rc, "feq_edge_sort")
    return perm, offsets, status


def block_diagonal_fwd(features, radial_table, distances, lvals_in, lvals_out, sh_scale, p1, p2,
                       num_bins, log_bins, mix="fp32"):
    lib = _require_cuda(features, radial_table, distances)
    features = _f32(features, "features")
    radial_table = _f32(radial_table, "radial_table")
    distances = _f32(distances, "distances")
    E, c_in, d_in = features.shape
    c_out = radial_table.shape[1]
    d_out = dim_of(lvals_out)
    if d_in != dim_of(lvals_in):
        raise ValueError(f"features dim {d_in} does not match lvals_in {list(lvals_in)}")
    if radial_table.shape[0] != num_bins + 1 or radial_table.shape[2] != c_in:
        raise ValueError(f"radial_table shape {tuple(radial_table.shape)} does not match "
                         f"(num_bins+1={num_bins + 1}, Cout, Cin={c_in}, W)")
    out = torch.empty(E, c_out, d_out, dtype=torch.float32, device=features.device)
    if E == 0:
        return out
    ai, ni = _lib.i32_array(lvals_in)
    ao, no = _lib.i32_array(lvals_out)
    mode = _lib.FEQ_MIX[mix]
    ws_bytes = lib.feq_block_diagonal_fwd_mix_workspace_bytes(E, c_in, c_out, ai, ni, ao, no, int(num_bins), mode)
    if ws_bytes == 0:
        raise RuntimeError("block-diagonal: unsupported layout (l <= 16, <= 64 irreps)")
    ws = _workspace(ws_bytes, features.device)
    rc = lib.feq_block_diagonal_fwd_mix(_p(features), _p(radial_table), _p(distances), E, c_in, c_out, ai, ni,
                                        ao, no, float(sh_scale), float(p1), float(p2), int(num_bins),
                                        int(bool(log_bins)), mode, _p(out), _p(ws), ws.numel(),
                                        _stream(features.device))
    _lib.check(rc, "feq_block_diagonal_fwd_mix")
    return out


def block_diagonal_bwd(grad_out, features, radial_table, distances, lvals_in, lvals_out, sh_scale, p1, p2,
                       num_bins, log_bins, mix="bf16x3"):
    """(grad_features, grad_table, grad_distances) of block_diagonal_fwd (tensor-core mixes in ``mix``)."""
    lib = _require_cuda(grad_out, features, radial_table, distances)
    grad_out = _f32(grad_out, "grad_output")
    features = _f32(features, "features")
    radial_table = _f32(radial_table, "radial_table")
    distances = _f32(distances, "distances")
    E, c_in, d_in = features.shape
    c_out = radial_table.shape[1]
    if grad_out.shape != (E, c_out, dim_of(lvals_out)):
        raise ValueError(f"grad_output shape {tuple(grad_out.shape)} does not match (E, Cout, d_out)")
    gf = torch.empty_like(features)
    gt = torch.empty_like(radial_table)
    gd = torch.empty(E, dtype=torch.float32, device=features.device)
    ai, ni = _lib.i32_array(lvals_in)
    ao, no = _lib.i32_array(lvals_out)
    mode = _lib.FEQ_MIX[mix]
    ws_bytes = lib.feq_block_diagonal_bwd_workspace_bytes(E, c_in, c_out, ai, ni, ao, no, int(num_bins), mode)
    if ws_bytes == 0:
        raise RuntimeError(f"block-diagonal backward: unsupported layout or mix {mix!r}")
    ws = _workspace(ws_bytes, features.device)
    rc = lib.feq_block_diagonal_bwd(_p(grad_out), _p(features), _p(radial_table), _p(distances), E, c_in, c_out, ai,
                                    ni, ao, no, float(sh_scale), float(p1), float(p2), int(num_bins),
                                    int(bool(log_bins)), mode, _p(gf), _p(gt), _p(gd), _p(ws), ws.numel(),
                                    _stream(features.device))
    _lib.check(rc, "feq_block_diagonal_bwd")
    return gf, gt, gd


def edgewise_fwd(x, distances, radial_table, lvals_in, lvals_out, c_out, sh_scale, p1, p2, num_bins,
                 log_bins, *, src=None, edge_add=None, directions=None, P=None, Q=None, status=None, mix="fp32"):
    """Fused Q . Lambda(r) . P^T . f.  Rows f[e] = x[src[e]] (+ edge_add[e]) or x[e].

    Basis from ``directions`` (E, 3) when given, else from the dense P (E, d_in, d_in)
    and Q (E, d_out, d_out).  ``mix``: "fp32" (CUDA cores), "bf16" (tensor cores,
    bf16 operands) or "bf16x3" (tensor cores, float32-level accuracy).
    """
    if mix not in _lib.FEQ_MIX:
        raise ValueError(f"mix must be one of {list(_lib.FEQ_MIX)}, got {mix!r}")
    lib = _require_cuda(x, distances, radial_table, src, edge_add, directions, P, Q)
    x = _f32(x, "x")
    distances = _f32(distances, "distances")
    radial_table = _f32(radial_table, "radial_table")
    E = distances.numel()
    c_in = x.shape[1]
    d_in, d_out = dim_of(lvals_in), dim_of(lvals_out)
    if x.shape[2] != d_in:
        raise ValueError(f"feature dim {x.shape[2]} does not match lvals_in {list(lvals_in)}")
    if radial_table.shape[0] != num_bins + 1 or radial_table.shape[1] != c_out or radial_table.shape[2] != c_in:
        raise ValueError(f"radial_table shape {tuple(radial_table.shape)} does not match "
                         f"({num_bins + 1}, {c_out}, {c_in}, W)")
    dev = x.device
    out = torch.empty(E, c_out, d_out, dtype=torch.float32, device=dev)
    if E == 0:
        return out
    args = _lib.FeqEdgewiseArgs()
    args.x = x.data_ptr()
    if src is not None:
        src = src.contiguous()
        if src.dtype != torch.int64:
            src = src.to(torch.int64)
        args.src = src.data_ptr()
        args.num_src_rows = x.shape[0]
    elif x.shape[0] != E:
        raise ValueError("edge features must have one row per edge")
    if edge_add is not None:
        edge_add = _f32(edge_add, "edge_features")
        args.edge_add = edge_add.data_ptr()
    if directions is not None:
        directions = _f32(directions, "directions")
        args.directions = directions.data_ptr()
    else:
        P = _f32(P, "P")
        Q = _f32(Q, "Q")
        if tuple(P.shape) != (E, d_in, d_in) or tuple(Q.shape) != (E, d_out, d_out):
            raise ValueError(f"P {tuple(P.shape)} / Q {tuple(Q.shape)} do not match E={E}, "
                             f"d_in={d_in}, d_out={d_out}")
        args.P_in = P.data_ptr()
        args.Q_out = Q.data_ptr()
    args.distances = distances.data_ptr()
    args.radial_table = radial_table.data_ptr()
    args.num_edges = E
    args.c_in, args.c_out = c_in, c_out
    ai, ni = _lib.i32_array(lvals_in)
    ao, no = _lib.i32_array(lvals_out)
    args.lvals_in, args.n_lvals_in = ai, ni
    args.lvals_out, args.n_lvals_out = ao, no
    args.sh_scale, args.bin_param1, args.bin_param2 = float(sh_scale), float(p1), float(p2)
    args.num_bins, args.log_bins = int(num_bins), int(bool(log_bins))
    args.out = out.data_ptr()
    if status is not None:
        args.status = status.data_ptr()
    args.mix_mode = _lib.FEQ_MIX[mix]
    ws_bytes = lib.feq_edgewise_workspace_bytes(ctypes.byref(args))
    if ws_bytes == 0:
        raise RuntimeError("edgewise: unsupported layout (l <= 16, <= 64 irreps, dim <= 512)")
    # Edges are independent, so a call whose scratch would exceed the cap runs as
    # consecutive edge ranges through one reused workspace (same results row by row).
    cap = EDGEWISE_WS_CAP or max(1 << 30, torch.cuda.get_device_properties(dev).total_memory // 8)
    if ws_bytes <= cap:
        ws = _workspace(ws_bytes, dev)
        rc = lib.feq_edgewise_fwd(ctypes.byref(args), _p(ws), ws.numel(), _stream(dev))
        _lib.check(rc, "feq_edgewise_fwd")
        return out
    n_chunks = -(-ws_bytes // cap)
    chunk = -(-E // n_chunks)
    chunk = -(-chunk // 128) * 128
    args.num_edges = chunk
    ws = _workspace(lib.feq_edgewise_workspace_bytes(ctypes.byref(args)), dev)
    row_in, row_out = c_in * d_in * 4, c_out * d_out * 4
    base = {f: getattr(args, f) for f in ("src", "x", "edge_add", "directions", "P_in", "Q_out", "distances", "out")}
    for e0 in range(0, E, chunk):
        n = min(chunk, E - e0)
        args.num_edges = n
        args.distances = base["distances"] + 4 * e0
        args.out = base["out"] + row_out * e0
        if src is not None:
            args.src = base["src"] + 8 * e0
        else:
            args.x = base["x"] + row_in * e0
        if edge_add is not None:
            args.edge_add = base["edge_add"] + row_in * e0
        if directions is not None:
            args.directions = base["directions"] + 12 * e0
        else:
            args.P_in = base["P_in"] + 4 * d_in * d_in * e0
            args.Q_out = base["Q_out"] + 4 * d_out * d_out * e0
        rc = lib.feq_edgewise_fwd(ctypes.byref(args), _p(ws), ws.numel(), _stream(dev))
        _lib.check(rc, "feq_edgewise_fwd")
    return out


def _separable_args(lvals_in, lvals_out, c_in, c_out, rank, mix):
    args = _lib.FeqSeparableArgs()
    ai, ni = _lib.i32_array(lvals_in)
    ao, no = _lib.i32_array(lvals_out)
    args.lvals_in, args.n_lvals_in = ai, ni
    args.lvals_out, args.n_lvals_out = ao, no
    args.c_in, args.c_out, args.rank = int(c_in), int(c_out), int(rank)
    args.mix_mode = _lib.FEQ_MIX.get(mix, -1)
    args.directions = 1          # the fused basis is the only one this kernel takes
    return args, (ai, ao)


def separable_supported(lvals_in, lvals_out, c_in, c_out, rank, mix) -> bool:
    """Whether feq_edgewise_separable_fwd runs this layer shape (else use edgewise_fwd)."""
    if mix not in ("bf16x3", "bf16"):
        return False
    args, _keep = _separable_args(lvals_in, lvals_out, c_in, c_out, rank, mix)
    return bool(_lib.load().feq_edgewise_separable_supported(ctypes.byref(args)))


def _aligned16(t):
    return t if t.data_ptr() % 16 == 0 else t.clone()


def edgewise_separable_fwd(x, distances, channel_patterns, radial_features, lvals_in, lvals_out, sh_scale, p1, p2,
                           num_bins, log_bins, *, directions, src=None, edge_add=None, status=None, mix="bf16x3"):
    """Q . Lambda(r) . P^T . f in one kernel for a separable radial table
    table[b, o, i, w] = sum_k channel_patterns[k, o, i] radial_features[b, k, w].

    Rows f[e] = x[src[e]] (+ edge_add[e]) or x[e]; basis from ``directions`` (E, 3).
    ``mix``: "bf16x3" (float32-level accuracy) or "bf16".  No workspace."""
    lib = _require_cuda(x, distances, channel_patterns, radial_features, src, edge_add, directions)
    x = _aligned16(_f32(x, "x"))
    distances = _f32(distances, "distances")
    cp = _f32(channel_patterns, "channel_patterns")
    rf = _aligned16(_f32(radial_features, "radial_features"))
    directions = _f32(directions, "directions")
    E = distances.numel()
    rank, c_out, c_in = cp.shape
    d_in, d_out = dim_of(lvals_in), dim_of(lvals_out)
    if x.shape[1] != c_in or x.shape[2] != d_in:
        raise ValueError(f"x {tuple(x.shape)} does not match (rows, {c_in}, {d_in})")
    if rf.shape[0] != num_bins + 1 or rf.shape[1] != rank:
        raise ValueError(f"radial_features {tuple(rf.shape)} does not match ({num_bins + 1}, {rank}, W)")
    dev = x.device
    out = torch.empty(E, c_out, d_out, dtype=torch.float32, device=dev)
    if E == 0:
        return out
    args, _keep = _separable_args(lvals_in, lvals_out, c_in, c_out, rank, mix)
    args.x = x.data_ptr()
    if src is not None:
        src = src.contiguous()
        if src.dtype != torch.int64:
            src = src.to(torch.int64)
        args.src = src.data_ptr()
        args.num_src_rows = x.shape[0]
    elif x.shape[0] != E:
        raise ValueError("edge features must have one row per edge")
    if edge_add is not None:
        edge_add = _aligned16(_f32(edge_add, "edge_features"))
        args.edge_add = edge_add.data_ptr()
    args.directions = directions.data_ptr()
    args.distances = distances.data_ptr()
    args.channel_patterns = cp.data_ptr()
    args.radial_features = rf.data_ptr()
    args.num_edges = E
    args.sh_scale, args.bin_param1, args.bin_param2 = float(sh_scale), float(p1), float(p2)
    args.num_bins, args.log_bins = int(num_bins), int(bool(log_bins))
    args.out = out.data_ptr()
    if status is not None:
        args.status = status.data_ptr()
    rc = lib.feq_edgewise_separable_fwd(ctypes.byref(args), _stream(dev))
    _lib.check(rc, "feq_edgewise_separable_fwd")
    return out


def segment_softmax(logits, perm, offsets, num_nodes):
    lib = _require_cuda(logits, perm, offsets)
    logits = _f32(logits, "logits")
    E, H = logits.shape
    w = torch.empty_like(logits)
    if E == 0:
        return w
    rc = lib.feq_segment_softmax(_p(logits), E, H, _p(perm), _p(offsets), int(num_nodes), _p(w),
                                 _stream(logits.device))
    _lib.check(rc, "feq_segment_softmax")
    return w


def edge_attention_weights(Q, K, scale, distances, decay, perm, offsets, num_nodes):
    lib = _require_cuda(Q, K, perm, offsets)
    Q, K = _f32(Q, "Q"), _f32(K, "K")
    E, H, D = Q.shape
    w = torch.empty(E, H, dtype=torch.float32, device=Q.device)
    if E == 0:
        return w
    dptr = None
    if decay is not None and distances is not None:
        distances = _f32(distances, "distances")
        dptr = _p(distances)
    rc = lib.feq_edge_attention_weights(_p(Q), _p(K), E, H, D, float(scale), dptr,
                                        float(decay) if dptr is not None else 0.0, _p(perm), _p(offsets),
                                        int(num_nodes), _p(w), _stream(Q.device))
    _lib.check(rc, "feq_edge_attention_weights")
    return w


def segment_pool(rows, perm, offsets, num_nodes, reduce="sum", weights=None):
    """rows (E, C, d) -> (N, C, d); optional per-head weights (E, H)."""
    lib = _require_cuda(rows, perm, offsets, weights)
    rows = _f32(rows, "edge_features")
    E = rows.shape[0]
    L = rows[0].numel() if E > 0 else int(torch.tensor(rows.shape[1:]).prod())
    if E == 0:   # every segment empty: sum, mean and max all give 0 (pooling.py:21-57)
        return torch.zeros((num_nodes,) + tuple(rows.shape[1:]), dtype=torch.float32, device=rows.device)
    out = torch.empty((num_nodes,) + tuple(rows.shape[1:]), dtype=torch.float32, device=rows.device)
    H = 0
    wptr = None
    if weights is not None:
        weights = _f32(weights, "weights")
        H = weights.shape[1]
        wptr = _p(weights)
    rc = lib.feq_segment_pool(_p(rows), L, wptr, H, _p(perm), _p(offsets), int(num_nodes),
                              _lib.FEQ_REDUCE[reduce], _p(out), _stream(rows.device))
    _lib.check(rc, "feq_segment_pool")
    return out


def attn_pool(qk, v, src, distances, perm, offsets, num_nodes, num_heads, scale, decay, reduce="sum",
              status=None, k=None):
    """Fused softmax-attention pooling: QK (N, 2C, d) node rows, V (E, Cv, dv) edge rows.

    With ``k`` given (partitioned graphs): ``qk`` holds only the destinations' Q rows
    (num_nodes, C, d) and ``k`` the K rows of every source node (N_src, C, d); src indexes k.
    """
    lib = _require_cuda(qk, v, src, perm, offsets)
    qk, v = _f32(qk, "QK"), _f32(v, "V")
    if k is not None:
        k = _f32(k, "K")
        if k.shape[1:] != qk.shape[1:]:
            raise ValueError(f"K rows {tuple(k.shape[1:])} do not match Q rows {tuple(qk.shape[1:])}")
        qk_rows = qk.shape[0]
        qk = qk.reshape(qk_rows, -1, qk.shape[-1])
    N, c2, d = qk.shape
    if k is not None:
        c2 = 2 * c2
    E, c_v, d_v = v.shape
    if E == 0:
        return torch.zeros(num_nodes, c_v, d_v, dtype=torch.float32, device=qk.device)
    out = torch.empty(num_nodes, c_v, d_v, dtype=torch.float32, device=qk.device)
    a = _lib.FeqAttnArgs()
    a.qk, a.v = qk.data_ptr(), v.data_ptr()
    src = src.contiguous()
    a.src = src.data_ptr()
    if decay is not None:
        distances = _f32(distances, "distances")
        a.distances = distances.data_ptr()
        a.decay_scale = float(decay)
    a.perm, a.offsets = perm.data_ptr(), offsets.data_ptr()
    a.num_nodes, a.num_edges = int(num_nodes), E
    a.c_qk, a.d_qk, a.c_v, a.d_v, a.num_heads = c2 // 2, d, c_v, d_v, int(num_heads)
    a.scale = float(scale)
    a.reduce = _lib.FEQ_REDUCE[reduce]
    a.out = out.data_ptr()
    if status is not None:
        a.status = status.data_ptr()
    if k is not None:
        a.k = k.data_ptr()
        a.num_src_nodes = int(k.shape[0])
    rc = lib.feq_attn_pool_fwd(ctypes.byref(a), _stream(qk.device))
    _lib.check(rc, "feq_attn_pool_fwd")
    return out


def attn_pool_bwd(grad_out, qk, v, src, dst, distances, perm, offsets, src_perm, src_offsets, num_nodes, num_heads,
                  scale, decay, reduce="sum", k=None, need_distances=False):
    """Backward of :func:`attn_pool` -> (grad_qk, grad_k, grad_v, grad_distances, grad_log_scale).

    Without ``k``: grad_qk has qk's shape (both the Q and the K halves) and grad_k is None.
    With ``k``: grad_qk is dL/dQ (num_nodes, C, d) and grad_k is dL/dk (N_src, C, d).
    grad_distances (the distance-decay term) is None unless ``need_distances``.
    ``src_perm`` / ``src_offsets``: :func:`edge_sort` of ``src`` over the source rows.
    """
    lib = _require_cuda(grad_out, qk, v, src, dst, perm, offsets, src_perm, src_offsets)
    qk, v, grad_out = _f32(qk, "QK"), _f32(v, "V"), _f32(grad_out, "grad_out")
    if k is not None:
        k = _f32(k, "K")
    E, c_v, d_v = v.shape
    N = int(num_nodes)
    d = qk.shape[-1]
    qrow = qk.shape[1] * d if k is not None else qk.shape[1] * d // 2
    dev = qk.device
    grad_qk = torch.empty_like(qk)
    grad_k = torch.empty_like(k) if k is not None else None
    grad_v = torch.empty_like(v)
    grad_d = torch.zeros(E, dtype=torch.float32, device=dev) if need_distances and decay is not None else None
    if E == 0:    # the forward is identically zero
        return (torch.zeros_like(qk), None if k is None else torch.zeros_like(k), grad_v, grad_d,
                torch.zeros((), dtype=torch.float32, device=dev))
    part = torch.empty(N, dtype=torch.float32, device=dev)
    scratch = torch.empty(max(2 * E * int(num_heads), 1), dtype=torch.float32, device=dev)
    b = _lib.FeqAttnBwdArgs()
    a = b.fwd
    src, dst = src.contiguous(), dst.contiguous()
    a.qk, a.v, a.src = qk.data_ptr(), v.data_ptr(), src.data_ptr()
    if decay is not None:
        distances = _f32(distances, "distances")
        a.distances = distances.data_ptr()
        a.decay_scale = float(decay)
    a.perm, a.offsets = perm.data_ptr(), offsets.data_ptr()
    a.num_nodes, a.num_edges = N, E
    a.c_qk, a.d_qk, a.c_v, a.d_v, a.num_heads = qrow // d, d, c_v, d_v, int(num_heads)
    a.scale = float(scale)
    a.reduce = _lib.FEQ_REDUCE[reduce]
    b.grad_out, b.dst = grad_out.data_ptr(), dst.data_ptr()
    b.src_perm, b.src_offsets = src_perm.data_ptr(), src_offsets.data_ptr()
    if k is not None:
        a.k = k.data_ptr()
        a.num_src_nodes = int(k.shape[0])
        b.grad_q, b.ldq = grad_qk.data_ptr(), qrow
        b.grad_k, b.ldk = grad_k.data_ptr(), qrow
    else:
        b.grad_q, b.ldq = grad_qk.data_ptr(), 2 * qrow
        b.grad_k, b.ldk = grad_qk.data_ptr() + 4 * qrow, 2 * qrow
    b.grad_v = grad_v.data_ptr()
    if grad_d is not None:
        b.grad_distances = grad_d.data_ptr()
    b.grad_scale_partial = part.data_ptr()
    b.edge_scratch = scratch.data_ptr()
    rc = lib.feq_attn_pool_bwd(ctypes.byref(b), _stream(dev))
    _lib.check(rc, "feq_attn_pool_bwd")
    return grad_qk, grad_k, grad_v, grad_d, part.sum()


def segment_softmax_bwd(weights, grad_weights, perm, offsets, num_nodes):
    lib = _require_cuda(weights, grad_weights, perm, offsets)
    weights, grad_weights = _f32(weights, "weights"), _f32(grad_weights, "grad_weights")
    E, H = weights.shape
    gl = torch.zeros_like(weights)
    if E == 0:
        return gl
    rc = lib.feq_segment_softmax_bwd(_p(weights), _p(grad_weights), E, H, _p(perm), _p(offsets), int(num_nodes),
                                     _p(gl), _stream(weights.device))
    _lib.check(rc, "feq_segment_softmax_bwd")
    return gl


def edge_attention_weights_bwd(grad_weights, weights, Q, K, scale, decay, perm, offsets, num_nodes,
                               need_distances=False):
    """Backward of :func:`edge_attention_weights` -> (grad_Q, grad_K, grad_distances, grad_log_scale)."""
    lib = _require_cuda(grad_weights, weights, Q, K, perm, offsets)
    Q, K = _f32(Q, "Q"), _f32(K, "K")
    weights, grad_weights = _f32(weights, "weights"), _f32(grad_weights, "grad_weights")
    E, H, D = Q.shape
    dev = Q.device
    gQ, gK = torch.zeros_like(Q), torch.zeros_like(K)
    gd = torch.zeros(E, dtype=torch.float32, device=dev) if need_distances and decay is not None else None
    part = torch.zeros(E, dtype=torch.float32, device=dev)
    if E == 0:
        return gQ, gK, gd, part.sum()
    gl = torch.empty(E, H, dtype=torch.float32, device=dev)
    rc = lib.feq_edge_attention_weights_bwd(_p(Q), _p(K), E, H, D, float(scale),
                                            float(decay) if decay is not None else 0.0, _p(perm), _p(offsets),
                                            int(num_nodes), _p(weights), _p(grad_weights), _p(gl), _p(gQ), _p(gK),
                                            _p(gd), _p(part), _stream(dev))
    _lib.check(rc, "feq_edge_attention_weights_bwd")
    return gQ, gK, gd, part.sum()


def segment_pool_bwd(grad_out, rows, out, dst, perm, offsets, num_nodes, reduce="sum", weights=None):
    """Backward of :func:`segment_pool` -> (grad_rows, grad_weights or None)."""
    lib = _require_cuda(grad_out, rows, dst, perm, offsets, weights)
    rows, grad_out = _f32(rows, "edge_features"), _f32(grad_out, "grad_out")
    E = rows.shape[0]
    grows = torch.zeros_like(rows)
    gw = None
    H = 0
    wptr = None
    if weights is not None:
        weights = _f32(weights, "weights")
        H = weights.shape[1]
        wptr = _p(weights)
        gw = torch.zeros_like(weights)
    if E == 0:
        return grows, gw
    L = rows[0].numel()
    ties = None
    if reduce == "max":
        out = _f32(out, "out")
        ties = torch.empty(int(num_nodes), L, dtype=torch.float32, device=rows.device)
    dst = dst.contiguous()
    rc = lib.feq_segment_pool_bwd(_p(rows), L, wptr, H, _p(dst), _p(perm), _p(offsets), int(num_nodes), E,
                                  _lib.FEQ_REDUCE[reduce], _p(out) if reduce == "max" else None, _p(grad_out),
                                  _p(ties), _p(grows), _p(gw), None, _stream(rows.device))
    _lib.check(rc, "feq_segment_pool_bwd")
    return grows, gw


def knn(coords, k, cell=None):
    """(N, k) int64 indices of the k nearest other points of every point (ascending
    distance, ties by index; -1 where fewer exist).  ``cell``: the cell side of the search
    grid (any positive value gives the same result); by default the median k-th neighbour
    distance of 64 sampled points."""
    lib = _require_cuda(coords)
    xyz = _f32(coords, "coordinates")
    if xyz.dim() != 2 or xyz.shape[1] != 3:
        raise ValueError("coordinates must have shape (N, 3)")
    N = xyz.shape[0]
    k = int(k)
    if not 1 <= k <= 64:
        raise ValueError("k must be in [1, 64]")
    nbr = torch.full((N, k), -1, dtype=torch.int64, device=xyz.device)
    if N < 2:
        return nbr
    lo = xyz.min(dim=0).values
    if cell is None:
        g = torch.Generator(device="cpu").manual_seed(0)
        sample = xyz[torch.randint(0, N, (min(64, N),), generator=g).to(xyz.device)]
        kk = min(k + 1, N)
        kth = torch.cdist(sample, xyz).topk(kk, dim=1, largest=False).values[:, -1]
        cell = float(kth.median())
        if not cell > 0.0:
            span = float((xyz.max(dim=0).values - lo).max())
            cell = span if span > 0.0 else 1.0
    status = torch.zeros(1, dtype=torch.int32, device=xyz.device)
    ws = _workspace(lib.feq_knn_workspace_bytes(N), xyz.device)
    x0, y0, z0 = (float(v) for v in lo.tolist())
    rc = lib.feq_knn_graph(_p(xyz), N, k, float(cell), x0, y0, z0, _p(nbr), _p(status), _p(ws), ws.numel(),
                           _stream(xyz.device))
    _lib.check(rc, "feq_knn_graph")
    if int(status.item()) != 0:
        raise RuntimeError("feq_knn_graph: search stopped before it was exact (cell too small)")
    return nbr


def radius_graph(coords, r, batch=None, loop=False):
    """(src, dst) int64 of every ordered pair of points of the same batch entry closer than
    ``r`` (strictly), without self pairs unless ``loop``; in (src, dst) order.  One host
    synchronisation (the edge count)."""
    lib = _require_cuda(coords, batch)
    xyz = _f32(coords, "coordinates")
    if xyz.dim() != 2 or xyz.shape[1] != 3:
        raise ValueError("coordinates must have shape (N, 3)")
    r = float(r)
    if not r > 0.0:
        raise ValueError(f"r must be > 0, got {r}")
    N = xyz.shape[0]
    dev = xyz.device
    empty = torch.empty(0, dtype=torch.int64, device=dev)
    if N == 0:
        return empty, empty
    if batch is not None:
        batch = batch.to(device=dev, dtype=torch.int64).contiguous()
        if batch.shape != (N,):
            raise ValueError(f"batch must have shape ({N},), got {tuple(batch.shape)}")
    lo = xyz.min(dim=0).values
    span = float((xyz.max(dim=0).values - lo).max())
    cell = max(r, span / 16000.0)           # <= 16384 cells per axis
    x0, y0, z0 = (float(v) - cell for v in lo.tolist())     # one empty cell of margin
    offsets = torch.empty(N + 1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _workspace(lib.feq_radius_workspace_bytes(N), dev)
    stream = _stream(dev)
    rc = lib.feq_radius_count(_p(xyz), _p(batch), N, r, int(bool(loop)), cell, x0, y0, z0, _p(offsets), _p(status),
                              _p(ws), ws.numel(), stream)
    _lib.check(rc, "feq_radius_count")
    E = int(offsets[N].item())
    if int(status.item()) != 0:
        raise RuntimeError("feq_radius_count: a point has a non-finite coordinate, lies outside the cell grid or "
                           "has a batch id out of range")
    src = torch.empty(E, dtype=torch.int64, device=dev)
    dst = torch.empty(E, dtype=torch.int64, device=dev)
    if E == 0:
        return src, dst
    pws = _workspace(lib.feq_radius_pairs_workspace_bytes(E), dev)
    rc = lib.feq_radius_fill(_p(xyz), _p(batch), N, r, int(bool(loop)), cell, x0, y0, z0, _p(offsets), E, _p(src),
                             _p(dst), _p(ws), ws.numel(), _p(pws), pws.numel(), stream)
    _lib.check(rc, "feq_radius_fill")
    return src, dst


# ---------------------------------------------------------------------------
# Node-level operators (forward)
# ---------------------------------------------------------------------------
def _node_rows(x, what):
    x = _f32(x, what)
    if x.dim() < 2:
        raise ValueError(f"{what} must have shape (..., C, d)")
    return x.reshape(-1, x.shape[-2], x.shape[-1])


def node_sep_layernorm(x, lvals, w_scalar, b_scalar, w_higher, eps):
    """SeparableEquivariantLayerNorm forward (see feq_node_sep_layernorm)."""
    lib = _require_cuda(x, w_scalar, b_scalar, w_higher)
    rows = _node_rows(x, "features")
    out = torch.empty_like(rows)
    arr, n = _lib.i32_array(lvals)
    c = lambda t: None if t is None else _f32(t, "weight")
    ws, bs, wh = c(w_scalar), c(b_scalar), c(w_higher)
    rc = lib.feq_node_sep_layernorm(_p(rows), rows.shape[0], rows.shape[1], arr, n, _p(ws), _p(bs), _p(wh),
                                    float(eps), _p(out), _stream(rows.device))
    _lib.check(rc, "feq_node_sep_layernorm")
    return out.view(x.shape)


def node_layernorm(x, lvals, ln_weight, ln_bias, ln_eps, rep_eps, eps):
    """EquivariantLayerNorm forward (see feq_node_layernorm); ln_weight None for mult 1."""
    lib = _require_cuda(x, ln_weight, ln_bias)
    rows = _node_rows(x, "features")
    out = torch.empty_like(rows)
    arr, n = _lib.i32_array(lvals)
    lw = None if ln_weight is None else _f32(ln_weight, "weight")
    lb = None if ln_bias is None else _f32(ln_bias, "bias")
    rc = lib.feq_node_layernorm(_p(rows), rows.shape[0], rows.shape[1], arr, n, _p(lw), _p(lb), float(ln_eps),
                                float(rep_eps), float(eps), _p(out), _stream(rows.device))
    _lib.check(rc, "feq_node_layernorm")
    return out.view(x.shape)


def node_rep_norm(x, lvals, eps):
    """RepNorm forward: (..., C, d) -> (..., C, n_irreps)."""
    lib = _require_cuda(x)
    rows = _node_rows(x, "features")
    arr, n = _lib.i32_array(lvals)
    norms = torch.empty(rows.shape[0], rows.shape[1], n, dtype=torch.float32, device=rows.device)
    rc = lib.feq_node_rep_norm(_p(rows), rows.shape[0], rows.shape[1], arr, n, float(eps), _p(norms),
                               _stream(rows.device))
    _lib.check(rc, "feq_node_rep_norm")
    return norms.view(*x.shape[:-1], n)


NODE_LINEAR_MIX = "bf16x3"      # tensor-core arithmetic of feq_node_linear_tc (float32-level accuracy)


def node_linear_tc_supported(lvals, c_in, c_out, mix=NODE_LINEAR_MIX) -> bool:
    """Whether feq_node_linear_tc serves this shape (else the three-step path)."""
    arr, n = _lib.i32_array(lvals)
    return _lib.load().feq_node_linear_tc_workspace_bytes(int(c_in), int(c_out), arr, n, _lib.FEQ_MIX[mix]) > 0


def node_linear(x, lvals, weight, bias, c_out, scalar_index):
    """EquivariantLinear forward (identity activation): (..., Cin, d) -> (..., Cout, d).

    One tensor-core kernel (feq_node_linear_tc, bf16x3) where it serves the shape; otherwise
    position-major layout kernels around one library GEMM per irrep.  ``scalar_index``: (d,)
    int8 device tensor, position -> bias column (-1 elsewhere)."""
    lib = _require_cuda(x, weight, bias)
    rows = _node_rows(x, "features")
    N, cin, d = rows.shape
    cout = int(c_out)
    dev = rows.device
    arr, n = _lib.i32_array(lvals)
    mode = _lib.FEQ_MIX[NODE_LINEAR_MIX]
    wsb = lib.feq_node_linear_tc_workspace_bytes(cin, cout, arr, n, mode)
    if wsb > 0:
        rows = _aligned16(rows)
        y = torch.empty(N, cout, d, dtype=torch.float32, device=dev)
        ws = _workspace(wsb, dev)
        w = _f32(weight, "weight").contiguous()
        b = None if bias is None else _f32(bias, "bias").contiguous()
        rc = lib.feq_node_linear_tc(_p(rows), N, cin, cout, arr, n, _p(w), _p(b), mode, _p(y), _p(ws), wsb, None,
                                    _stream(dev))
        _lib.check(rc, "feq_node_linear_tc")
        return y.view(*x.shape[:-2], cout, d)
    xt = torch.empty(d, N, cin, dtype=torch.float32, device=dev)
    rc = lib.feq_node_to_posmajor(_p(rows), N, cin, d, _p(xt), _stream(dev))
    _lib.check(rc, "feq_node_to_posmajor")
    yt = torch.empty(d, N, cout, dtype=torch.float32, device=dev)
    w = _f32(weight, "weight").view(len(lvals), cout, cin)
    off = 0
    for r, l in enumerate(lvals):
        k = 2 * int(l) + 1
        torch.matmul(xt[off:off + k].view(k * N, cin), w[r].t(), out=yt[off:off + k].view(k * N, cout))
        off += k
    y = torch.empty(N, cout, d, dtype=torch.float32, device=dev)
    arr, n = _lib.i32_array(lvals)
    b = None if bias is None else _f32(bias, "bias")
    rc = lib.feq_node_from_posmajor(_p(yt), N, cout, arr, n, _p(b), _p(scalar_index) if b is not None else None,
                                    _p(y), _stream(dev))
    _lib.check(rc, "feq_node_from_posmajor")
    return y.view(*x.shape[:-2], cout, d)


RADIAL_MAX_FREQS, RADIAL_MAX_HIDDEN = 64, 256     # limits of feq_radial_features


def radial_features(bin_edges, min_val, max_val, frequencies, w1, b1, w2, b2, w3, b3):
    """SeparableRadialNet's features at the bin edges in one launch (feq_radial_features):
    sinusoid x envelope basis, two SiLU layers and the head, weights as nn.Linear holds them.
    Returns (num_edges, out_dim) float32."""
    lib = _require_cuda(bin_edges, frequencies, w1, b1, w2, b2, w3, b3)
    edges = _f32(bin_edges, "bin_edges")
    tensors = [_f32(t, n) for t, n in ((frequencies, "frequencies"), (w1, "w1"), (b1, "b1"), (w2, "w2"),
                                       (b2, "b2"), (w3, "w3"), (b3, "b3"))]
    freqs, w1, b1, w2, b2, w3, b3 = tensors
    hidden, out_dim = w1.shape[0], w3.shape[0]
    out = torch.empty(edges.numel(), out_dim, dtype=torch.float32, device=edges.device)
    rc = lib.feq_radial_features(_p(edges), edges.numel(), float(min_val), float(max_val), _p(freqs), freqs.numel(),
                                 _p(w1), _p(b1), hidden, _p(w2), _p(b2), _p(w3), _p(b3), out_dim, _p(out),
                                 _stream(edges.device))
    _lib.check(rc, "feq_radial_features")
    return out


def dense_linear_tc_supported(m, k, mix=NODE_LINEAR_MIX) -> bool:
    """Whether feq_dense_linear_tc serves y = x w^T + b with w (m, k)."""
    return _lib.load().feq_dense_linear_tc_workspace_bytes(int(m), int(k), _lib.FEQ_MIX[mix]) > 0


def dense_linear(x, weight, bias=None, mix=NODE_LINEAR_MIX):
    """nn.Linear forward y = x w^T + b on the tensor cores (feq_dense_linear_tc, bf16x3 by
    default); x (..., k), weight (m, k).  Raises for shapes the kernel does not serve."""
    lib = _require_cuda(x, weight, bias)
    m, k = weight.shape
    xx = _aligned16(_f32(x, "x").reshape(-1, k).contiguous())
    n = xx.shape[0]
    dev = xx.device
    y = torch.empty(n, m, dtype=torch.float32, device=dev)
    mode = _lib.FEQ_MIX[mix]
    wsb = lib.feq_dense_linear_tc_workspace_bytes(m, k, mode)
    ws = _workspace(wsb, dev)
    w = _f32(weight, "weight").contiguous()
    b = None if bias is None else _f32(bias, "bias").contiguous()
    rc = lib.feq_dense_linear_tc(_p(xx), n, m, k, _p(w), _p(b), mode, _p(y), _p(ws), wsb, None, _stream(dev))
    _lib.check(rc, "feq_dense_linear_tc")
    return y.view(*x.shape[:-1], m)


def node_gate(x, z, lvals):
    """x * sigmoid(z)[..., c, irrep(position)]; z (..., C * n_irreps)."""
    lib = _require_cuda(x, z)
    rows = _node_rows(x, "features")
    z = _f32(z, "gate")
    out = torch.empty_like(rows)
    arr, n = _lib.i32_array(lvals)
    if z.numel() != rows.shape[0] * rows.shape[1] * n:
        raise ValueError("gate pre-activation has the wrong size")
    rc = lib.feq_node_gate(_p(rows), _p(z), rows.shape[0], rows.shape[1], arr, n, _p(out), _stream(rows.device))
    _lib.check(rc, "feq_node_gate")
    return out.view(x.shape)


def profile_enable(on: bool = True) -> None:
    """Start (or stop) recording CUDA-event stage timings inside the native library."""
    _lib.load().feq_profile_enable(1 if on else 0)


def profile_read() -> dict:
    """{stage: (total_ms, launches)} of the stages recorded since profile_enable(True)."""
    lib = _lib.load()
    n = lib.feq_profile_read(-1, None, 0, None, None)
    if n < 0:
        _lib.check(-n, "feq_profile_read")
    out = {}
    for i in range(n):
        buf = ctypes.create_string_buffer(64)
        ms, cnt = ctypes.c_double(), ctypes.c_int64()
        lib.feq_profile_read(i, buf, 64, ctypes.byref(ms), ctypes.byref(cnt))
        out[buf.value.decode()] = (ms.value, cnt.value)
    return out
