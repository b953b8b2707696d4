"""vmap rules of the custom operators: the vmapped dimension joins the pairs.

Every operator of this package treats dim 0 of its tensors as a batch of
independent pairs, so ``torch.func.vmap`` over V slices of a batch of B pairs
is one native call over V * B pairs.  The rule moves the vmapped dimension to
the front, expands unbatched pair tensors, merges it with the pair dimension,
calls the operator once, and splits the pair dimension of each result again.

One kind of tensor does not lead with pairs: the DP's saved stream, an opaque
byte buffer laid out per warp of the launch plan.  The operators that return
it round its size up to a multiple of their pair count, so after a call over
V * B pairs it reshapes to [V, bytes / V] (and to [V1, V2, ...] under nested
vmaps, since V1 * V2 divides the pair count too).  A backward that receives
the buffer batched flattens it back to the one buffer the forward wrote.  A
backward that receives it unbatched while its gradients are batched comes
from an unbatched forward with vmapped cotangents (``torch.func.jacrev``,
``vjp`` under vmap): it runs once per slice on the same saved state.

The reference registers one fold rule per operator
(hibana2077/torchwarp src/torchwarp/udtw/_ops.py:77-90); its saved tensors are
pair-leading, which the saved stream here is not.
"""

from typing import Iterable

import torch
from torch import Tensor


def round_to_pairs(nbytes: int, pairs: int) -> int:
    """Size of a saved-stream buffer: ``nbytes`` rounded up to a multiple of
    ``pairs`` (the vmap rules split the buffer by any divisor of the pair
    count)."""
    if pairs <= 1:
        return nbytes
    return (nbytes + pairs - 1) // pairs * pairs


def _as_tuple(out):
    """(results as a tuple, whether the op returns a tuple)."""
    return ((out,), False) if isinstance(out, Tensor) else (tuple(out), True)


def register_fold_rule(op, flat_in: Iterable[int] = (), flat_out: Iterable[int] = (),
                       placeholder_out: Iterable[int] = ()):
    """Register the fold rule on a torch.library custom op.

    flat_in / flat_out: argument / result positions that hold a saved-stream
    byte buffer.  placeholder_out: result positions that may be an empty [0]
    tensor standing for "no such output" (not a batch of zero pairs)."""
    flat_in, flat_out = frozenset(flat_in), frozenset(flat_out)
    placeholder_out = frozenset(placeholder_out)

    def rule(info, in_dims, *args):
        V = info.batch_size
        is_t = [isinstance(a, Tensor) for a in args]
        flat_unbatched = any(is_t[k] and in_dims[k] is None for k in flat_in if k < len(args))
        if flat_unbatched:
            return _loop(op, V, in_dims, args)
        folded, pairs = [], None
        for k, (a, d) in enumerate(zip(args, in_dims)):
            if is_t[k]:
                if k in flat_in:
                    a = a.movedim(d, 0).reshape(-1)
                else:
                    a = a.movedim(d, 0) if d is not None else a.expand(V, *a.shape)
                    a = a.reshape(V * a.shape[1], *a.shape[2:])
                    pairs = a.shape[0] if pairs is None else pairs
            folded.append(a)
        out, multi = _as_tuple(op(*folded))
        res, dims = [], []
        for i, o in enumerate(out):
            if i in flat_out:
                res.append(o.reshape(V, -1))
                dims.append(0)
            elif i in placeholder_out and o.dim() == 1 and o.numel() == 0 and pairs:
                res.append(o)
                dims.append(None)
            else:
                res.append(o.reshape(V, o.shape[0] // V, *o.shape[1:]))
                dims.append(0)
        if multi:
            return tuple(res), tuple(dims)
        return res[0], dims[0]

    op.register_vmap(rule)


def _loop(op, V, in_dims, args):
    """One call per vmap slice (saved state shared by every slice)."""
    per = []
    for v in range(V):
        sl = [a.select(d, v) if isinstance(a, Tensor) and d is not None else a
              for a, d in zip(args, in_dims)]
        per.append(_as_tuple(op(*sl)))
    multi = per[0][1]
    outs = tuple(torch.stack([p[0][i] for p in per]) for i in range(len(per[0][0])))
    if multi:
        return outs, tuple(0 for _ in outs)
    return outs[0], 0
