"""Autograd for the attention and pooling operators: native forward, native backward.

The reference differentiates its scatter / gather formulation with PyTorch autograd
(flash_eq/layers/attention.py:92-167, flash_eq/layers/pooling.py:21-57).  Here each
operator is one ``torch.autograd.Function`` whose forward and backward are the
library's segment kernels (``feq_attn_pool_fwd`` / ``feq_attn_pool_bwd``,
``feq_edge_attention_weights`` / ``..._bwd``, ``feq_segment_softmax`` / ``..._bwd``,
``feq_segment_pool`` / ``..._bwd``).  The backward kernels reduce over dst- and
src-sorted segments in a fixed order, so gradients are bitwise reproducible.

Without autograd (inference, or no input requiring grad) each entry point calls the
forward op directly.
"""
from __future__ import annotations

import torch

from . import ops


def _tracks(*tensors) -> bool:
    return torch.is_grad_enabled() and any(torch.is_tensor(t) and t.requires_grad for t in tensors)


def _d(t):
    return None if t is None else t.detach()


# ---------------------------------------------------------------------------
# Fused attention pooling (EquivariantAttention)
# ---------------------------------------------------------------------------
class _AttnPool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qk, v, distances, log_scale, k, graph, num_heads, scale, decay, reduce):
        perm, offsets = graph.dst_segments()
        out = ops.attn_pool(qk, v, graph.src, distances, perm, offsets, graph.num_nodes, num_heads, scale, decay,
                            reduce, k=k)
        ctx.save_for_backward(qk, v, distances, k)
        ctx.cfg = (graph, num_heads, scale, decay, reduce)
        ctx.has_distances = distances is not None
        ctx.has_k = k is not None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        qk, v, distances, k = ctx.saved_tensors
        if not ctx.has_distances:
            distances = None
        if not ctx.has_k:
            k = None
        graph, num_heads, scale, decay, reduce = ctx.cfg
        perm, offsets = graph.dst_segments()
        src_perm, src_offsets = graph.src_segments()
        need_d = ctx.has_distances and ctx.needs_input_grad[2]
        gqk, gk, gv, gd, gls = ops.attn_pool_bwd(grad_out, qk, v, graph.src, graph.dst, distances, perm, offsets,
                                                 src_perm, src_offsets, graph.num_nodes, num_heads, scale, decay,
                                                 reduce, k=k, need_distances=need_d)
        return (gqk if ctx.needs_input_grad[0] else None, gv if ctx.needs_input_grad[1] else None,
                gd if need_d else None, gls if ctx.needs_input_grad[3] else None,
                gk if ctx.needs_input_grad[4] else None, None, None, None, None, None)


def attn_pool(qk, v, distances, log_scale, graph, num_heads, scale, decay, reduce, k=None):
    """softmax-attention pooling of V onto each destination (see ``ops.attn_pool``), with autograd
    for qk, v, distances (decay term), log_scale (``scale`` = exp(log_scale) as a float) and k."""
    if decay is None:
        distances = None
    if _tracks(qk, v, distances, log_scale, k):
        return _AttnPool.apply(qk, v, distances, log_scale, k, graph, num_heads, scale, decay, reduce)
    perm, offsets = graph.dst_segments()
    return ops.attn_pool(_d(qk), _d(v), graph.src, _d(distances), perm, offsets, graph.num_nodes, num_heads, scale,
                         decay, reduce, k=_d(k))


# ---------------------------------------------------------------------------
# Edge-level attention weights (EquivariantEdgeAttention)
# ---------------------------------------------------------------------------
class _EdgeAttentionWeights(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, distances, log_scale, graph, scale, decay):
        perm, offsets = graph.dst_segments()
        w = ops.edge_attention_weights(Q, K, scale, distances, decay, perm, offsets, graph.num_nodes)
        ctx.save_for_backward(Q, K, w)
        ctx.cfg = (graph, scale, decay)
        ctx.has_distances = distances is not None
        return w

    @staticmethod
    def backward(ctx, grad_w):
        Q, K, w = ctx.saved_tensors
        graph, scale, decay = ctx.cfg
        perm, offsets = graph.dst_segments()
        need_d = ctx.has_distances and ctx.needs_input_grad[2]
        gQ, gK, gd, gls = ops.edge_attention_weights_bwd(grad_w, w, Q, K, scale, decay, perm, offsets,
                                                         graph.num_nodes, need_distances=need_d)
        return (gQ if ctx.needs_input_grad[0] else None, gK if ctx.needs_input_grad[1] else None,
                gd if need_d else None, gls if ctx.needs_input_grad[3] else None, None, None, None)


def edge_attention_weights(Q, K, distances, log_scale, graph, scale, decay):
    """(E, H, D) Q and K -> (E, H) softmax weights over each destination's in-edges."""
    if decay is None:
        distances = None
    if _tracks(Q, K, distances, log_scale):
        return _EdgeAttentionWeights.apply(Q, K, distances, log_scale, graph, scale, decay)
    perm, offsets = graph.dst_segments()
    return ops.edge_attention_weights(_d(Q), _d(K), scale, _d(distances), decay, perm, offsets, graph.num_nodes)


# ---------------------------------------------------------------------------
# Segment softmax of given logits
# ---------------------------------------------------------------------------
class _SegmentSoftmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, perm, offsets, num_nodes):
        w = ops.segment_softmax(logits, perm, offsets, num_nodes)
        ctx.save_for_backward(w, perm, offsets)
        ctx.num_nodes = num_nodes
        return w

    @staticmethod
    def backward(ctx, grad_w):
        w, perm, offsets = ctx.saved_tensors
        return ops.segment_softmax_bwd(w, grad_w, perm, offsets, ctx.num_nodes), None, None, None


def segment_softmax(logits, perm, offsets, num_nodes):
    if _tracks(logits):
        return _SegmentSoftmax.apply(logits, perm, offsets, num_nodes)
    return ops.segment_softmax(_d(logits), perm, offsets, num_nodes)


# ---------------------------------------------------------------------------
# Segment pooling (GraphPooling)
# ---------------------------------------------------------------------------
class _SegmentPool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, weights, graph, reduce):
        perm, offsets = graph.dst_segments()
        out = ops.segment_pool(rows, perm, offsets, graph.num_nodes, reduce, weights)
        ctx.save_for_backward(rows, weights, out if reduce == "max" else None)
        ctx.cfg = (graph, reduce)
        ctx.has_w = weights is not None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        rows, weights, out = ctx.saved_tensors
        graph, reduce = ctx.cfg
        if not ctx.has_w:
            weights = None
        perm, offsets = graph.dst_segments()
        grows, gw = ops.segment_pool_bwd(grad_out, rows, out, graph.dst, perm, offsets, graph.num_nodes, reduce,
                                         weights)
        return (grows if ctx.needs_input_grad[0] else None,
                gw if (ctx.has_w and ctx.needs_input_grad[1]) else None, None, None)


def segment_pool(rows, graph, reduce="sum", weights=None):
    if _tracks(rows, weights):
        return _SegmentPool.apply(rows, weights, graph, reduce)
    perm, offsets = graph.dst_segments()
    return ops.segment_pool(_d(rows), perm, offsets, graph.num_nodes, reduce, _d(weights))
