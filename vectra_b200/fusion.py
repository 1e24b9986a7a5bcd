"""An opt-in Inductor pass for models served with this library's operator.

The reference's compile pass (compiler/vectra_compiler/replacement.py:
193-235) cuts the matched eager chain at the value operand of its final
batched matmul, so the operator receives `reshape(V_BMM)`: the
contiguous copy of V that the eager `weights @ v` needed
(`clone(expand(permute(view(...))))` in the post-grad graph). This
library's kernels read any strided view in place, so the copy is pure
overhead: one extra read and write of V per attention site (13 us per site
of the price model at 1,024 targets on a B200).

`value_views_pass` rewires each `vectra.rbf_attention` call to the tensor
the copy was made from, when the chain between them only moves the same
elements (reshapes, `expand` to the same shape, a `clone`) and that tensor
has no broadcast (stride-0) dimension; the copy then has no user and
Inductor drops it. The operator reads the same values as before, bit for
bit (its kernels take strided views); the model's other kernels may be
generated differently once the copy is gone, so a compiled model's outputs
agree within rounding. The reference's pass itself is untouched: this pass
runs after it, as Inductor's post-grad custom pass.

    from vectra_b200 import fusion
    with fusion.installed():
        compiled, report = backend.compile_for_serving(model, inputs, n)
"""

import contextlib

import torch

aten = torch.ops.aten

# Ops through which a value-preserving chain may run from the view to the
# operator's value argument.
_VIEW_OPS = {aten.reshape.default, aten.view.default, aten._unsafe_view.default}
_COPY_OPS = {aten.clone.default}
_EXPAND_OPS = {aten.expand.default}


def _shape(node):
    val = node.meta.get('val') if hasattr(node, 'meta') else None
    return tuple(val.shape) if isinstance(val, torch.Tensor) else None


def _source_view(v):
    """The tensor node whose elements `v` holds, in the same shape, if v is
    reached from it only through a copy and views that restore its shape
    (an `expand` to the same shape is looked through); else None."""
    target_shape = _shape(v)
    node, copied = v, False
    while True:
        is_call = isinstance(node, torch.fx.Node) and node.op == 'call_function'
        if (copied and _shape(node) == target_shape and
                not (is_call and node.target in _EXPAND_OPS)):
            return node
        if not is_call:
            return None
        if node.target in _VIEW_OPS:
            node = node.args[0]
        elif node.target in _COPY_OPS:
            if set(node.kwargs) - {'memory_format'}:
                return None
            copied = True
            node = node.args[0]
        elif node.target in _EXPAND_OPS:
            # An expand that changes nothing (same shape) is a no-op view.
            src = node.args[0]
            if _shape(src) != _shape(node):
                return None
            node = src
        else:
            return None


def value_views_pass(graph: torch.fx.Graph) -> int:
    """Rewires every vectra.rbf_attention's value argument to the view its
    copy was made from (see the module docstring); returns the number of
    calls rewired."""
    rewired = 0
    op = torch.ops.vectra.rbf_attention.default
    for node in list(graph.nodes):
        if node.op != 'call_function' or node.target is not op:
            continue
        v = node.args[2]
        if not isinstance(v, torch.fx.Node):
            continue
        src = _source_view(v)
        if src is None or src is v:
            continue
        val = src.meta.get('val')
        if not isinstance(val, torch.Tensor) or val.dtype != v.meta['val'].dtype:
            continue
        # A broadcast view (stride 0 over a dimension longer than 1) stays
        # behind its copy: tensor-map kernels take no zero strides.
        if any(st == 0 and sz > 1 for st, sz in zip(val.stride(), val.shape)):
            continue
        node.args = node.args[:2] + (src,) + node.args[3:]
        rewired += 1
    if rewired:
        graph.eliminate_dead_code()
    return rewired


class _Pass:
    """Inductor's post-grad custom pass: value_views_pass with a count."""

    def __init__(self):
        self.rewired = 0

    def __call__(self, graph):
        self.rewired += value_views_pass(graph)

    def uuid(self):  # Inductor's pass-cache key
        return 'vectra_b200.fusion.value_views_pass.v1'


@contextlib.contextmanager
def installed():
    """Installs value_views_pass as Inductor's post-grad custom pass for the
    block (compiles inside it rewire the operator's value argument); yields
    the pass, whose `rewired` counts the calls rewired."""
    from torch._inductor import config as inductor_config  # pylint: disable=import-outside-toplevel
    p = _Pass()
    with inductor_config.patch(post_grad_custom_post_pass=p):
        yield p
