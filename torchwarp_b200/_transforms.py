"""Helpers that keep the autograd Functions usable under torch.compile and
torch.func.

* ``traceable(cls)``: Dynamo traces a ``torch.autograd.Function`` (into one
  graph with ``fullgraph=True``) only when the class defines no custom
  ``jvp``.  The Functions of this package that have a native forward-mode
  rule get a twin without it, returned here and used through ``pick`` while
  Dynamo is tracing; eager calls keep the rule.  Forward-mode AD inside a
  compiled region is the one thing the twin cannot do.
* ``once_differentiable``: torch's decorator of that name marks a backward
  that must not be differentiated again by wrapping its results in an error
  node, which needs ``requires_grad`` set on plain tensors and fails on the
  wrapped tensors of torch.func transforms (jacrev runs the backward under
  vmap with grad mode on).  Under torch.func this version computes the
  backward without recording it and passes its results through
  ``_NotTwice``, a Function that depends on one differentiable input of the
  backward and raises if a second derivative ever reaches it, so the
  semantics stay the same: first order works, second order raises.  While
  Dynamo traces the backward it runs as it is.
"""

import functools

import torch


def traceable(cls):
    """``cls`` without its custom jvp (a subclass; everything else shared)."""
    return type(cls.__name__ + "Traced", (cls,),
                {"jvp": staticmethod(torch.autograd.Function.jvp),
                 "__doc__": cls.__doc__, "__module__": cls.__module__})


def pick(cls, twin):
    """The Function to apply: the traceable twin under torch.compile."""
    return twin if torch.compiler.is_compiling() else cls


class _NotTwice(torch.autograd.Function):
    """Identity on the results of a first-order-only backward, tied to one of
    its differentiable inputs; differentiating through it raises."""

    generate_vmap_rule = True

    @staticmethod
    def forward(anchor, *outs):
        return tuple(o.clone() for o in outs)

    @staticmethod
    def setup_context(ctx, inputs, output):
        pass

    @staticmethod
    def backward(ctx, *grads):
        raise RuntimeError("trying to differentiate twice a function that was marked "
                           "once-differentiable (a first-order native backward)")


def once_differentiable(fn):
    wrapped = torch.autograd.function.once_differentiable(fn)

    @functools.wraps(fn)
    def wrapper(ctx, *args):
        if torch.compiler.is_compiling():
            return fn(ctx, *args)
        if not torch._C._are_functorch_transforms_active():
            return wrapped(ctx, *args)
        with torch.no_grad():
            out = fn(ctx, *args)
        if not torch.is_grad_enabled():
            return out
        anchors = [t for t in (*args, *ctx.saved_tensors)
                   if isinstance(t, torch.Tensor) and t.requires_grad]
        if not anchors:
            return out
        outs = out if isinstance(out, tuple) else (out,)
        idx = [i for i, o in enumerate(outs) if isinstance(o, torch.Tensor)]
        guarded = _NotTwice.apply(anchors[0], *[outs[i] for i in idx])
        res = list(outs)
        for i, g in zip(idx, guarded):
            res[i] = g
        return tuple(res) if isinstance(out, tuple) else res[0]

    return wrapper
