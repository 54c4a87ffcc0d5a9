"""TEST INFRASTRUCTURE ONLY -- CPU restatement of flash-eq's edge-message path.

This module is the parity checker for the B200 implementation and the timed
CPU baseline ("reference arm").  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / ``--impl reference`` legs may import it.  The
product package never does.

Every function restates one piece of hmblair/flash-eq and cites where:

* ``m_first_perm``          flash_eq/representations/wigner.py:243-272
* ``weight_dim``            flash_eq/representations/types.py:157-172, 345-347
* ``block_layout``          flash_eq/cuda/csrc/block_diagonal.cu:1191-1266 (via C)
* ``real_generators``       flash_eq/representations/types.py:74-135
* ``wigner_basis``          flash_eq/representations/wigner.py:144-240, 341-370
* ``binning``               flash_eq/cuda/csrc/block_diagonal.cu:82-115 (via C)
* ``block_diagonal_fwd``    flash_eq/cuda/csrc/block_diagonal.cu:558-733 (via C),
                            flash_eq/cuda/block_diagonal.py:206-274
* ``edgewise_fwd``          flash_eq/layers/linear.py:100-160
* ``radial_table``          flash_eq/layers/radial.py:242-275
* ``binning_params``        flash_eq/layers/radial.py:277-283
* ``edge_attention``        flash_eq/layers/attention.py:72-167
* ``pool``                  flash_eq/layers/pooling.py:21-57

Pinned by ``tests/test_oracle_pins.py`` against fixtures produced by importing
the reference itself (``tests/golden/make_golden.py``).  The block-diagonal
restatement has no CPU counterpart in the reference; it is pinned by the
reference's own equivariance and self-loop properties on CPU and, on the GPU
box, by the reference's CUDA kernel compiled into ``oracle/_ref``.
"""
from __future__ import annotations

import ctypes
import math
import os
from functools import lru_cache

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_bd.so")
MAX_L = 17  # block_diagonal.cu:172


# ----------------------------------------------------------------------------
# C restatement loader
# ----------------------------------------------------------------------------
@lru_cache(maxsize=1)
def _stale() -> bool:
    if not os.path.isfile(_LIB_PATH):
        return True
    built = os.path.getmtime(_LIB_PATH)
    return any(os.path.getmtime(os.path.join(_HERE, f)) > built
               for f in ("block_diagonal_ref.c", "block_diagonal_bwd_ref.c"))


def _lib() -> ctypes.CDLL:
    if _stale():
        import subprocess

        subprocess.check_call(["make", "-s", "-C", _HERE], stdout=subprocess.DEVNULL)
    lib = ctypes.CDLL(_LIB_PATH)
    i32p = ctypes.POINTER(ctypes.c_int)
    for name, fp in (("oracle_bd_fwd_f32", ctypes.c_void_p), ("oracle_bd_fwd_f64", ctypes.c_void_p)):
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [fp, fp, fp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                       ctypes.c_int, ctypes.c_int, i32p, ctypes.c_int, i32p, ctypes.c_int,
                       ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                       fp, ctypes.c_int]
    lib.oracle_block_layout.restype = ctypes.c_int
    lib.oracle_block_layout.argtypes = [i32p, ctypes.c_int, i32p, ctypes.c_int, i32p, i32p, i32p]
    lib.oracle_binning_f32.restype = None
    lib.oracle_binning_f32.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    lib.oracle_num_cpus.restype = ctypes.c_int
    vp = ctypes.c_void_p
    lib.oracle_bd_bwd_f64.restype = ctypes.c_int
    lib.oracle_bd_bwd_f64.argtypes = [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, i32p, ctypes.c_int, i32p, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                      vp, vp, vp]
    return lib


def num_cpus() -> int:
    return int(_lib().oracle_num_cpus())


def _i32arr(vals):
    arr = (ctypes.c_int * max(1, len(vals)))(*[int(v) for v in vals])
    return arr


# ----------------------------------------------------------------------------
# Representation bookkeeping (integer, bit-exact)
# ----------------------------------------------------------------------------
def m_first_perm(lvals) -> np.ndarray:
    """Standard (l, m) order -> m-first order (wigner.py:243-272).

    Position list: every m=0 component (irreps in list order), then for
    m = 1..lmax and each irrep with l >= m the pair (+m, -m).
    """
    lvals = [int(x) for x in lvals]
    offs = np.cumsum([0] + [2 * l + 1 for l in lvals])
    perm = [int(offs[i] + l) for i, l in enumerate(lvals)]
    for m in range(1, (max(lvals) if lvals else 0) + 1):
        for i, l in enumerate(lvals):
            if l >= m:
                perm.append(int(offs[i] + l + m))
                perm.append(int(offs[i] + l - m))
    return np.asarray(perm, dtype=np.int64)


def weight_dim(lvals_in, lvals_out) -> int:
    """ProductRepr.nreps(): sum over irrep pairs of (2 min(l1, l2) + 1) (types.py:157-172,345-347)."""
    return int(sum(2 * min(a, b) + 1 for a in lvals_in for b in lvals_out))


def block_layout(lvals_in, lvals_out):
    """precompute_block_info (block_diagonal.cu:1191-1266) -> (mmax, params[m]=(m,n_in,n_out,in_off,out_off,w_off))."""
    p = (ctypes.c_int * (MAX_L * 6))()
    li = (ctypes.c_int * (MAX_L * MAX_L))()
    lo = (ctypes.c_int * (MAX_L * MAX_L))()
    mmax = _lib().oracle_block_layout(_i32arr(lvals_in), len(lvals_in), _i32arr(lvals_out),
                                      len(lvals_out), p, li, lo)
    if mmax < 0:
        raise RuntimeError("mmax exceeds the reference limit (MAX_LVALS=17)")
    params = np.frombuffer(p, dtype=np.int32).reshape(MAX_L, 6)[: mmax + 1].copy()
    return mmax, params


# ----------------------------------------------------------------------------
# Wigner-D basis (reference algorithm: batched matrix exponential)
# ----------------------------------------------------------------------------
def _raising(l):
    m = np.arange(-l, l)
    return np.diag(-np.sqrt(l * (l + 1) - m * (m + 1.0)), k=-1)


def _lowering(l):
    m = np.arange(-l + 1, l + 1)
    return np.diag(np.sqrt(l * (l + 1) - m * (m - 1.0)), k=1)


def _toreal(l):
    """Complex -> real SH change of basis (types.py:114-135)."""
    n = 2 * l + 1
    q = np.zeros((n, n), dtype=np.complex128)
    s2 = 2 ** -0.5
    for m in range(-l, 0):
        q[l + m, l + abs(m)] = s2
        q[l + m, l - abs(m)] = -1j * s2
    for m in range(1, l + 1):
        q[l + m, l + abs(m)] = (-1) ** m * s2
        q[l + m, l - abs(m)] = 1j * (-1) ** m * s2
    q[l, l] = 1
    return (-1j) ** l * q


def real_generators(l: int, dtype=np.float32) -> np.ndarray:
    """so(3) generators in the real-SH basis ordered [Lz, Lx, Ly] (types.py:86-112).

    Rounded to float32 exactly as the reference stores them (REAL_DTYPE).
    """
    rp = _raising(l).astype(np.complex128)
    lw = _lowering(l).astype(np.complex128)
    jx = 0.5 * (rp + lw)
    jy = -0.5j * (rp - lw)
    jz = 1j * np.diag(np.arange(-l, l + 1).astype(np.complex128))
    q = _toreal(l)
    qh = q.conj().T
    lx = (qh @ jx @ q).real
    lz = (qh @ jy @ q).real
    ly = (qh @ jz @ q).real
    return np.stack([lz, lx, ly]).astype(dtype)


def repr_generators(lvals) -> torch.Tensor:
    dims = [2 * int(l) + 1 for l in lvals]
    d = sum(dims)
    g = np.zeros((3, d, d), dtype=np.float32)
    off = 0
    for l, n in zip(lvals, dims):
        g[:, off:off + n, off:off + n] = real_generators(int(l))
        off += n
    return torch.from_numpy(g)


def rot(axis: torch.Tensor, angle: torch.Tensor, lvals) -> torch.Tensor:
    """WignerD.rot (wigner.py:144-196): matrix_exp(angle * axis @ gens), nan->0, l=0 := 1."""
    gens = repr_generators(lvals).to(axis.dtype)
    d = gens.shape[-1]
    *b, _ = axis.shape
    K = angle[..., None, None] * (axis @ gens.view(3, -1)).view(*b, d, d)
    r = torch.nan_to_num(torch.linalg.matrix_exp(K), 0.0)
    off = 0
    for l in lvals:
        if int(l) == 0:
            r[..., off, off] = 1.0
        off += 2 * int(l) + 1
    return r


def wigner_basis(directions: torch.Tensor, lvals) -> torch.Tensor:
    """WignerDBasis.forward for one repr (wigner.py:198-240, 341-370), on CPU."""
    eps = 1e-8 if directions.dtype not in (torch.float16, torch.bfloat16) else 1e-5
    d = directions / (torch.linalg.norm(directions, dim=-1, keepdim=True) + eps)
    axis = torch.stack([-d[..., 1], d[..., 0], torch.zeros_like(d[..., 0])], dim=-1)
    axis = axis / (torch.linalg.norm(axis, dim=-1, keepdim=True) + eps)
    angle = torch.arccos(d[..., 2].clamp(-1 + eps, 1 - eps))
    m_std = rot(axis, angle, lvals)          # rot_to_ez(...).mT.mT
    perm = torch.from_numpy(m_first_perm(lvals))
    return m_std[..., perm]


# ----------------------------------------------------------------------------
# Binning and the block-diagonal mix (C restatement)
# ----------------------------------------------------------------------------
def binning_params(num_bins, min_val, max_val, log):
    """SeparableRadialNet.binning_params (radial.py:277-283, with :500-501 for log)."""
    if log:
        log_min = torch.tensor(min_val).log().item()
        inv_log_range = 1.0 / (torch.tensor(max_val / min_val).log().item())
        return log_min, inv_log_range
    return min_val, num_bins / (max_val - min_val)


def binning(dist: np.ndarray, p1, p2, num_bins, log_bins):
    dist = np.ascontiguousarray(dist, dtype=np.float32)
    lo = np.empty(dist.shape[0], dtype=np.int32)
    t = np.empty(dist.shape[0], dtype=np.float32)
    _lib().oracle_binning_f32(dist.ctypes.data, dist.shape[0], p1, p2, num_bins, int(bool(log_bins)),
                              lo.ctypes.data, t.ctypes.data)
    return lo, t


def block_diagonal_fwd(features, table, dist, lvals_in, lvals_out, sh_scale, p1, p2,
                       num_bins, log_bins, nthreads=None):
    """block_diagonal_cuda forward on CPU (block_diagonal.py:206-274, block_diagonal.cu:558-733).

    features (E, Cin, Din) m-first; table (num_bins+1, Cout, Cin, Wdim); dist (E,).
    float32 or float64 inputs.  Distances are cast to the feature dtype first
    (block_diagonal.py:260).  Sorting by distance does not change the result.
    """
    as_torch = isinstance(features, torch.Tensor)
    f = features.detach().cpu().numpy() if as_torch else np.asarray(features)
    tb = table.detach().cpu().numpy() if isinstance(table, torch.Tensor) else np.asarray(table)
    ds = dist.detach().cpu().numpy() if isinstance(dist, torch.Tensor) else np.asarray(dist)
    dt = np.float64 if f.dtype == np.float64 else np.float32
    f = np.ascontiguousarray(f, dtype=dt)
    tb = np.ascontiguousarray(tb, dtype=dt)
    ds = np.ascontiguousarray(ds.astype(dt))
    E, Cin, Din = f.shape
    Cout, Wdim = tb.shape[1], tb.shape[3]
    Dout = sum(2 * int(l) + 1 for l in lvals_out)
    out = np.empty((E, Cout, Dout), dtype=dt)
    fn = _lib().oracle_bd_fwd_f64 if dt == np.float64 else _lib().oracle_bd_fwd_f32
    if E > 0:
        rc = fn(f.ctypes.data, tb.ctypes.data, ds.ctypes.data, E, Cin, Cout, Din, Dout, Wdim,
                _i32arr(lvals_in), len(lvals_in), _i32arr(lvals_out), len(lvals_out),
                float(sh_scale), float(p1), float(p2), int(num_bins), int(bool(log_bins)),
                out.ctypes.data, int(nthreads or num_cpus()))
        if rc < 0:
            raise RuntimeError("oracle block-diagonal: unsupported layout")
    return torch.from_numpy(out) if as_torch else out


def block_diagonal_bwd(grad_out, features, table, dist, lvals_in, lvals_out, sh_scale, p1, p2, num_bins,
                       log_bins):
    """block_diagonal_cuda backward on CPU in float64 (block_diagonal.cu:747-1161):
    (grad_features, grad_table, grad_distances) as float64 torch tensors."""
    c = lambda x: np.ascontiguousarray((x.detach().cpu().numpy() if isinstance(x, torch.Tensor) else x),
                                       dtype=np.float64)
    go, f, tb, ds = c(grad_out), c(features), c(table), c(dist)
    E, Cin, Din = f.shape
    Cout, Wdim = tb.shape[1], tb.shape[3]
    Dout = go.shape[2]
    gf = np.empty_like(f)
    gt = np.empty_like(tb)
    gd = np.empty(E, dtype=np.float64)
    rc = _lib().oracle_bd_bwd_f64(go.ctypes.data, f.ctypes.data, tb.ctypes.data, ds.ctypes.data, E, Cin, Cout,
                                  Din, Dout, Wdim, _i32arr(lvals_in), len(lvals_in), _i32arr(lvals_out),
                                  len(lvals_out), float(sh_scale), float(p1), float(p2), int(num_bins),
                                  int(bool(log_bins)), gf.ctypes.data, gt.ctypes.data, gd.ctypes.data)
    if rc < 0:
        raise RuntimeError("oracle block-diagonal backward: unsupported layout")
    return torch.from_numpy(gf), torch.from_numpy(gt), torch.from_numpy(gd)


def edgewise_fwd(P, Q, edge_features, distances, table, lvals_in, lvals_out, sh_scale,
                 p1, p2, num_bins, log_bins, nthreads=None):
    """EquivariantEdgewiseLinear.forward (linear.py:100-160) on CPU tensors."""
    f_diag = torch.bmm(edge_features, P)
    out_diag = block_diagonal_fwd(f_diag, table, distances, lvals_in, lvals_out, sh_scale,
                                  p1, p2, num_bins, log_bins, nthreads)
    return torch.bmm(out_diag, Q.mT)


# ----------------------------------------------------------------------------
# Radial table (reference SeparableRadialNet.forward, from its parameters)
# ----------------------------------------------------------------------------
def radial_table(state: dict, num_bins, min_val, max_val, log, rank, weight_dim_,
                 prefix: str = "") -> torch.Tensor:
    """Binned table (num_bins+1, Cout, Cin, Wdim) from a SeparableRadialNet state dict (radial.py:242-275)."""
    g = lambda k: state[prefix + k].double()
    if log:
        edges = torch.logspace(math.log10(min_val), math.log10(max_val), num_bins + 1,
                               dtype=torch.float32).double()
    else:
        edges = torch.linspace(min_val, max_val, num_bins + 1, dtype=torch.float32).double()
    x = ((edges - min_val) / (max_val - min_val)).clamp(0.0, 1.0)
    env = 1.0 - 10.0 * x ** 3 + 15.0 * x ** 4 - 6.0 * x ** 5
    ang = x[:, None] * g("frequencies")[None, :]
    basis = torch.cat([torch.sin(ang) * env[:, None], torch.cos(ang) * env[:, None]], dim=-1)
    h = torch.nn.functional.silu(basis @ g("trunk.0.weight").T + g("trunk.0.bias"))
    h = torch.nn.functional.silu(h @ g("trunk.2.weight").T + g("trunk.2.bias"))
    f = (h @ g("head.weight").T + g("head.bias")).view(-1, rank, weight_dim_)
    return torch.einsum("koi,bkw->boiw", g("channel_patterns"), f)


# ----------------------------------------------------------------------------
# Attention and pooling
# ----------------------------------------------------------------------------
def segment_softmax(logits: torch.Tensor, dst: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """_neighbor_softmax (attention.py:108-141): amax, exp, sum, divide by (sum + 1e-8)."""
    E, H = logits.shape
    idx = dst.view(-1, 1).expand(E, H)
    mx = torch.full((num_nodes, H), float("-inf"), dtype=logits.dtype)
    mx.scatter_reduce_(0, idx, logits, reduce="amax", include_self=False)
    ex = torch.exp(logits - mx.gather(0, idx))
    sm = torch.zeros(num_nodes, H, dtype=logits.dtype).scatter_add_(0, idx, ex)
    return ex / (sm.gather(0, idx) + 1e-8)


def edge_attention(Qe, Ke, V, dst, num_nodes, scale, num_heads, distances=None,
                   distance_decay_scale=None):
    """EquivariantEdgeAttention.forward (attention.py:72-167), dropout off."""
    logits = (Qe * Ke).sum(-1) * scale
    if distance_decay_scale is not None and distances is not None:
        logits = logits - distances.unsqueeze(-1) / distance_decay_scale
    w = segment_softmax(logits, dst, num_nodes)
    E, mult, dim = V.shape
    if num_heads == 1:
        return V * w.view(E, 1, 1)
    return (V.view(E, num_heads, mult // num_heads, dim) * w.view(E, num_heads, 1, 1)).view(E, mult, dim)


def pool(edge_features: torch.Tensor, dst: torch.Tensor, num_nodes: int, reduce: str = "sum"):
    """GraphPooling sum / mean / max (pooling.py:21-57)."""
    _, c, d = edge_features.shape
    idx = dst.view(-1, 1, 1).expand(-1, c, d)
    if reduce == "max":
        out = torch.full((num_nodes, c, d), float("-inf"), dtype=edge_features.dtype)
        out.scatter_reduce_(0, idx, edge_features, reduce="amax")
        return out.nan_to_num(neginf=0.0)
    out = torch.zeros(num_nodes, c, d, dtype=edge_features.dtype).scatter_add_(0, idx, edge_features)
    if reduce == "mean":
        cnt = torch.zeros(num_nodes, dtype=edge_features.dtype)
        cnt.scatter_add_(0, dst, torch.ones_like(dst, dtype=edge_features.dtype))
        out = out / cnt.clamp(min=1).view(-1, 1, 1)
    return out
