"""vectra_b200.fusion's value-views pass, on CPU.

After the reference's compile pass rewrites an attention site, the
operator's value argument is the contiguous copy the eager bmm needed
(compiler/vectra_compiler/replacement.py:205-213). The pass hands the
operator the view the copy was made from instead; the operator's values
must not change (on CPU the whole compiled model stays bit-identical), and
chains that are not pure copies are left alone.
"""

import shutil

import pytest
import torch

from tests import reference_swap
from vectra_b200 import fusion

aten = torch.ops.aten


def _graph_with_value(chain):
    """An FX graph: x [2, 3, 5, 4] -> chain -> vectra.rbf_attention(q, q,
    v, scale) with v the chain's result; returns (graph, rbf node, x)."""
    g = torch.fx.Graph()
    x = g.placeholder('x')
    x.meta['val'] = torch.empty(2, 3, 5, 4)
    s = g.placeholder('s')
    s.meta['val'] = torch.empty(1, 3, 1, 1)
    v = chain(g, x)
    rbf = g.call_function(torch.ops.vectra.rbf_attention.default,
                          (x, x, v, s, None))
    g.output(rbf)
    return g, rbf, x


def _node(g, target, args, shape, **kwargs):
    n = g.call_function(target, args, kwargs)
    n.meta['val'] = torch.empty(shape)
    return n


def test_contiguity_copy_is_bypassed():
    def chain(g, x):
        e = _node(g, aten.expand.default, (x, [2, 3, 5, 4]), (2, 3, 5, 4))
        c = _node(g, aten.clone.default, (e,), (2, 3, 5, 4),
                  memory_format=torch.contiguous_format)
        r = _node(g, aten.reshape.default, (c, [6, 5, 4]), (6, 5, 4))
        return _node(g, aten.reshape.default, (r, [2, 3, 5, 4]),
                     (2, 3, 5, 4))
    g, rbf, x = _graph_with_value(chain)
    assert fusion.value_views_pass(g) == 1
    assert rbf.args[2] is x
    # The copy and its views had no other user: gone.
    assert not any(n.target is aten.clone.default for n in g.nodes)


def _val(shape, strides):
    return torch.empty_strided(shape, strides)


@pytest.mark.parametrize('kind', ['no_copy', 'broadcast', 'reorders'])
def test_other_chains_are_left_alone(kind):
    def chain(g, x):
        if kind == 'no_copy':  # already a view: nothing to bypass
            r = _node(g, aten.reshape.default, (x, [6, 5, 4]), (6, 5, 4))
            return _node(g, aten.reshape.default, (r, [2, 3, 5, 4]),
                         (2, 3, 5, 4))
        if kind == 'broadcast':  # the copy materialises a stride-0 view
            sl = _node(g, aten.slice.Tensor, (x, 1, 0, 1), (2, 1, 5, 4))
            e = g.call_function(aten.expand.default, (sl, [2, 3, 5, 4]))
            e.meta['val'] = _val((2, 3, 5, 4), (60, 0, 4, 1))
            return _node(g, aten.clone.default, (e,), (2, 3, 5, 4))
        # The copy's source holds the elements in another order.
        t = _node(g, aten.permute.default, (x, [0, 1, 3, 2]), (2, 3, 4, 5))
        c = _node(g, aten.clone.default, (t,), (2, 3, 4, 5))
        return _node(g, aten.reshape.default, (c, [2, 3, 5, 4]),
                     (2, 3, 5, 4))
    g, rbf, x = _graph_with_value(chain)
    before = rbf.args[2]
    assert fusion.value_views_pass(g) == 0
    assert rbf.args[2] is before


def test_copy_of_a_computed_tensor_is_bypassed():
    # clone(mul(x, 2)) holds mul's values: the operator reads mul directly.
    def chain(g, x):
        m = _node(g, aten.mul.Tensor, (x, 2.0), (2, 3, 5, 4))
        return _node(g, aten.clone.default, (m,), (2, 3, 5, 4))
    g, rbf, _ = _graph_with_value(chain)
    assert fusion.value_views_pass(g) == 1
    assert rbf.args[2].target is aten.mul.Tensor


@pytest.mark.skipif(not reference_swap.installed(),
                    reason='the reference is not installed in baseline/_ref')
def test_reference_model_compiled_with_the_pass_is_bit_identical():
    from torch._inductor import config as inductor_config  # pylint: disable=import-outside-toplevel
    # Inductor's CPU backend compiles and links OpenMP C++; the system
    # compiler is the one whose OpenMP spec files are complete.
    system_gxx = shutil.which('g++', path='/usr/bin')
    cxx = {'cpp.cxx': (None, system_gxx)} if system_gxx else {}
    with inductor_config.patch(cxx):
        _compile_and_compare()


def _compile_and_compare():
    ref = reference_swap.load_reference()
    cfg = ref.model.ModelConfig(embedding_dim=32, attribute_dim=8,
                                d_model=64, num_heads=2, num_layers=2,
                                ffn_dim=128, num_candidates=16)
    torch.manual_seed(0)
    model = ref.model.PriceTransformer(cfg).eval()
    model.set_block_dtype(torch.bfloat16)
    inputs = tuple(ref.model.example_inputs(cfg, 4))
    torch._dynamo.reset()  # pylint: disable=protected-access
    plain, report = ref.backend.compile_for_serving(model, inputs, 2)
    torch._dynamo.reset()  # pylint: disable=protected-access
    with fusion.installed() as p:
        fused, report2 = ref.backend.compile_for_serving(model, inputs, 2)
    assert report.sites == report2.sites == 2
    assert p.rewired == 2
    with torch.no_grad():
        for seed in (1, 2):
            x = tuple(ref.model.example_inputs(cfg, 4, seed=seed))
            assert torch.equal(plain(*x), fused(*x))
