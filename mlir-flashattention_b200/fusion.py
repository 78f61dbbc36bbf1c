"""The reference's fusion pass for PyTorch graphs.

``fuse_attention(gm)`` is FuseAttentionPattern (lib/Attention/FusionPass.cpp:95-168)
restated for ``torch.fx`` graphs: it finds the unfused attention chain

    scores = Q @ Kᵀ            QKᵀ           (FusionPass.cpp:138-145)
    scores = scores * scale     scale         (:76-88, :147-150)
    scores = mask ? -inf : scores   [mask]    (:117-124)
    P = softmax(scores, dim=-1) softmax       (:106-112)
    O = P @ V                   P·V, anchor   (:95-104)

and replaces it with one call of ``attention_fused(Q, K, V, scale, mask)``,
which runs ``attention.fused`` on the tensor cores (``fused`` in this
package).  Like the reference pattern it is anchored on the P·V matmul and
walks the chain backwards: the softmax that writes P, then the op that
writes the softmax input (a mask select when it has a mask operand, else the
scale), then the scale, then the QKᵀ product whose operands are Q and K.
The scale is the scalar operand of the multiplication (a division by a
constant d gives 1/d).

Where the reference matches any generic by its operand count, the graph
pass checks what each op computes: a matmul against a transposed K (the
last two dims swapped), a multiplication or division by a Python number,
a select of -inf (or the most negative float, as in the reference's
test/Attention/fusion.mlir) where the mask is True, and a softmax over the
last dim.  Unlike the reference, which erases the five ops even when other
ops read their buffers, a chain is only rewritten when each intermediate
(scores, scaled and masked scores, P) has no other user; the intermediates
then become dead and are removed.
"""
from __future__ import annotations

import math
import operator

import torch
import torch.fx

__all__ = ["attention_fused", "fuse_attention", "fuse"]

_NEG_LIMIT = -3.4028234663852886e38  # -FLT_MAX: the reference test's "-inf"


def attention_fused(q, k, v, scale, mask=None):
    """The op the pass emits: ``attention.fused ins(q, k, v) scale(scale)
    [mask(mask)]`` with a freshly allocated output (bf16 for bf16 / e4m3
    inputs, f16 for f16, f32 for f32), as returned by this package's
    ``fused``.  ``mask`` is bool with True = masked.

    A traced graph carries no shapes, so the pass cannot check ranks: any
    leading dims shared by q, k and v (and a mask over them, or a [Nq, Nk]
    one) are flattened into the head dim of ``fused``'s [1, H, N, D] form,
    and the result takes q's shape back."""
    from . import fused  # noqa: PLC0415  (the package imports this module lazily)
    q4, k4, v4, m4, lead = _as_4d(q, k, v, mask)
    out = fused(q4, k4, v4, float(scale), mask=m4)
    return out if lead is None else out.reshape(*lead, *out.shape[-2:])


def _as_4d(q, k, v, mask):
    """q, k, v (and the mask) in a rank ``fused`` takes, and q's leading dims
    to restore (None when nothing was reshaped)."""
    from . import VerifyError  # noqa: PLC0415

    if q.dim() in (2, 4) and k.dim() == q.dim() and v.dim() == q.dim() and \
            (mask is None or mask.dim() in (2, q.dim())):
        return q, k, v, mask, None
    lead = tuple(q.shape[:-2])
    if q.dim() < 2 or tuple(k.shape[:-2]) != lead or tuple(v.shape[:-2]) != lead:
        raise VerifyError("attention.fused: Q, K and V need the same leading dims "
                          "(rank 2 or 4 otherwise)")
    h = 1
    for d in lead:
        h *= d
    q4, k4, v4 = (t.reshape(1, h, *t.shape[-2:]) for t in (q, k, v))
    m4 = mask
    if mask is not None and mask.dim() > 2:
        if tuple(mask.shape[:-2]) != lead:
            raise VerifyError("attention.fused: the mask must be [seq_q, seq_k] or share "
                              "Q's leading dims")
        m4 = mask.reshape(1, h, *mask.shape[-2:])
    return q4, k4, v4, m4, lead


_MATMULS = {operator.matmul, torch.matmul, torch.bmm}
_MATMUL_METHODS = {"matmul", "bmm", "__matmul__"}
_SOFTMAXES = {torch.softmax, torch.nn.functional.softmax, torch.special.softmax}
_MULS = {operator.mul, torch.mul}
_DIVS = {operator.truediv, torch.div, torch.true_divide}


def _is_fn(n, targets):
    return isinstance(n, torch.fx.Node) and n.op == "call_function" and n.target in targets


def _is_method(n, names):
    return isinstance(n, torch.fx.Node) and n.op == "call_method" and n.target in names


def _arg(n, i, name, default=None):
    if len(n.args) > i:
        return n.args[i]
    return n.kwargs.get(name, default)


def _single_user(n, user):
    return isinstance(n, torch.fx.Node) and list(n.users) == [user]


def _matmul_operands(n):
    """(a, b) of a matmul node, else None."""
    if _is_fn(n, _MATMULS) and len(n.args) == 2 and not n.kwargs:
        return n.args[0], n.args[1]
    if _is_method(n, _MATMUL_METHODS) and len(n.args) == 2 and not n.kwargs:
        return n.args[0], n.args[1]
    return None


def _rank(n):
    meta = n.meta.get("tensor_meta") if isinstance(n, torch.fx.Node) else None
    return len(meta.shape) if meta is not None and hasattr(meta, "shape") else None


def _last_two(dims, rank):
    """True when the dims (a transpose's pair) are the last two of a tensor."""
    norm = set()
    for d in dims:
        if not isinstance(d, int):
            return False
        if d < 0:
            norm.add(d)
        elif rank is not None:
            norm.add(d - rank)
        else:
            return False
    return norm == {-2, -1}


def _untransposed(n):
    """K when ``n`` is K with its last two dims swapped, else None."""
    if not isinstance(n, torch.fx.Node):
        return None
    if _is_method(n, {"transpose", "swapaxes", "swapdims"}) and len(n.args) == 3:
        k = n.args[0]
        return k if _last_two(n.args[1:], _rank(k)) else None
    if _is_fn(n, {torch.transpose, torch.swapaxes, torch.swapdims}) and len(n.args) == 3:
        k = n.args[0]
        return k if _last_two(n.args[1:], _rank(k)) else None
    if _is_method(n, {"t"}) and len(n.args) == 1:
        return n.args[0]
    if n.op == "call_function" and n.target is getattr and len(n.args) == 2:
        base, attr = n.args
        if attr == "mT" or (attr == "T" and _rank(base) == 2):
            return base
    if _is_method(n, {"permute"}) and len(n.args) >= 2:
        dims = n.args[1] if len(n.args) == 2 and isinstance(n.args[1], (list, tuple)) else n.args[1:]
        r = len(dims)
        if list(dims) == list(range(r - 2)) + [r - 1, r - 2] or \
                list(dims) == list(range(-r, -2)) + [-1, -2]:
            return n.args[0]
    return None


def _softmax_input(n):
    """The input of a softmax over the last dim, else None."""
    if _is_fn(n, _SOFTMAXES):
        x, dim = _arg(n, 0, "input"), _arg(n, 1, "dim")
        if _arg(n, 3 if n.target is torch.nn.functional.softmax else 2, "dtype") is not None:
            return None
    elif _is_method(n, {"softmax"}):
        x, dim = n.args[0], _arg(n, 1, "dim")
        if n.kwargs.get("dtype") is not None:
            return None
    else:
        return None
    if dim == -1 or (isinstance(dim, int) and _rank(x) is not None and dim == _rank(x) - 1):
        return x
    return None


def _is_neg_inf(v):
    return isinstance(v, (int, float)) and (v == -math.inf or v <= _NEG_LIMIT)


def _mask_select(n):
    """(scores, mask, negate) of a select that puts -inf where the mask says so
    (negate: the mask marks the kept entries, as in ``where(keep, s, -inf)``),
    else None."""
    if _is_method(n, {"masked_fill"}) and len(n.args) == 3 and not n.kwargs:
        s, m, val = n.args
        return (s, m, False) if _is_neg_inf(val) else None
    if _is_fn(n, {torch.masked_fill}) and len(n.args) == 3 and not n.kwargs:
        s, m, val = n.args
        return (s, m, False) if _is_neg_inf(val) else None
    if _is_fn(n, {torch.where}) and len(n.args) == 3 and not n.kwargs:
        c, a, b = n.args
        if _is_neg_inf(a) and isinstance(b, torch.fx.Node):
            return b, c, False
        if _is_neg_inf(b) and isinstance(a, torch.fx.Node):
            return a, c, True
    return None


def _scale_op(n):
    """(scores, scale) of a multiplication or division by a Python number,
    else None (FusionPass.cpp:76-88 takes the first mulf's outer operand)."""
    if _is_fn(n, _MULS) or _is_method(n, {"mul", "__mul__"}):
        if len(n.args) != 2 or n.kwargs:
            return None
        a, b = n.args
        if isinstance(a, torch.fx.Node) and isinstance(b, (int, float)):
            return a, float(b)
        if isinstance(b, torch.fx.Node) and isinstance(a, (int, float)):
            return b, float(a)
        return None
    if _is_fn(n, _DIVS) or _is_method(n, {"div", "__truediv__", "true_divide"}):
        if len(n.args) != 2 or n.kwargs:
            return None
        a, b = n.args
        if isinstance(a, torch.fx.Node) and isinstance(b, (int, float)) and b != 0:
            return a, 1.0 / float(b)
    return None


def _match(pv):
    """The chain anchored on the P·V matmul ``pv`` as (Q, K, V, scale, mask,
    negate_mask, chain nodes from softmax back to Kᵀ), or None
    (FuseAttentionPattern::matchAndRewrite steps 1-5)."""
    ops = _matmul_operands(pv)
    if ops is None:
        return None
    probs, v = ops                                   # step 1
    if not _single_user(probs, pv):
        return None
    x = _softmax_input(probs)                        # step 2
    if not _single_user(x, probs):
        return None
    mask, negate = None, False
    sel = _mask_select(x)                            # step 3: mask, then scale
    if sel is not None:
        scaled, mask, negate = sel
        if not _single_user(scaled, x) or not isinstance(mask, torch.fx.Node):
            return None
    else:
        scaled = x
    sc = _scale_op(scaled)
    if sc is None:
        return None
    qk, scale = sc
    if not _single_user(qk, scaled):
        return None
    qk_ops = _matmul_operands(qk)                    # step 4: QKᵀ
    if qk_ops is None:
        return None
    q, kt = qk_ops
    k = _untransposed(kt)
    if k is None or not isinstance(q, torch.fx.Node):
        return None
    chain = [probs] + ([x] if sel is not None else []) + [scaled, qk, kt]
    return q, k, v, scale, mask, negate, chain       # step 5: the scale value


def fuse_attention(gm: torch.fx.GraphModule) -> int:
    """Rewrite every unfused attention chain of ``gm`` into one
    ``attention_fused`` call (step 6 of the reference pattern) and recompile;
    returns the number of chains rewritten."""
    graph = gm.graph
    count = 0
    for pv in list(graph.nodes):
        if pv.graph is not graph:  # erased by an earlier rewrite
            continue
        m = _match(pv)
        if m is None:
            continue
        q, k, v, scale, mask, negate, chain = m
        with graph.inserting_before(pv):
            if mask is not None and negate:
                mask = graph.call_function(torch.logical_not, (mask,))
            fused_node = graph.call_function(attention_fused, (q, k, v, scale, mask))
        fused_node.meta.update(pv.meta)
        pv.replace_all_uses_with(fused_node)
        # Erase the anchor, then the chain back to QKᵀ (uses before defs, as
        # the reference erases its five ops); Kᵀ only when nothing else reads it.
        graph.erase_node(pv)
        for n in chain:
            if not n.users:
                graph.erase_node(n)
        count += 1
    if count:
        graph.lint()
        gm.recompile()
    return count


def fuse(fn) -> torch.fx.GraphModule:
    """Trace ``fn`` (an ``nn.Module`` or a function of tensors) with
    ``torch.fx.symbolic_trace`` and run ``fuse_attention`` on the graph."""
    gm = torch.fx.symbolic_trace(fn)
    fuse_attention(gm)
    return gm
