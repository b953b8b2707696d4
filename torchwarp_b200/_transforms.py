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
  vmap with grad mode on).  Under torch.func (and while Dynamo traces the
  backward) this version runs the backward as it is: its results come from the native custom operators, which have no
  autograd formula, so differentiating them again raises all the same.
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


def once_differentiable(fn):
    wrapped = torch.autograd.function.once_differentiable(fn)

    @functools.wraps(fn)
    def wrapper(ctx, *args):
        if torch.compiler.is_compiling() or torch._C._are_functorch_transforms_active():
            return fn(ctx, *args)
        return wrapped(ctx, *args)

    return wrapper
