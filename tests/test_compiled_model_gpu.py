"""benchmark config 5: the reference's compile pass rewrites a model's
attention to this library's operator, inside one graph.

The reference's `vectra_compiler` (installed unmodified into baseline/_ref;
skipped when it is not there) imports `vectra_kernels.custom_ops` only to
register the operator (compiler/vectra_compiler/replacement.py:38-39).
Binding that module name to `vectra_b200.custom_ops` is the whole
integration (the one-file swap of kernels/vectra_kernels/custom_ops.py);
the pass's replacement graph then calls this library's
torch.ops.vectra.rbf_attention. `compile_for_serving`
(compiler/vectra_compiler/backend.py:98-136) proves one graph and counts
the rewritten sites. The model (tests/spatial_model.py) writes its
attention as the eager RBF chain, as the price model does.
"""

import pytest
import torch

from tests import spatial_model
from tests.conftest import compile_pass_installed

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(
        not compile_pass_installed(),
        reason='the reference compile pass is not installed in baseline/_ref'),
]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _compile(backend, model, args, sites):
    torch._dynamo.reset()  # pylint: disable=protected-access
    return backend.compile_for_serving(model, args, expected_sites=sites)


def _launches_per_forward(compiled, args):
    import vectra_b200  # pylint: disable=import-outside-toplevel
    with torch.no_grad():
        before = vectra_b200.launch_count()
        out = compiled(*args)
        torch.cuda.synchronize()
    return vectra_b200.launch_count() - before, out


def test_bf16_model_every_site_rewritten_in_one_graph(backend):
    torch.manual_seed(0)
    m32 = spatial_model.SpatialNet(layers=3).cuda().eval()
    model = spatial_model.SpatialNet(layers=3).cuda().eval()
    model.load_state_dict(m32.state_dict())
    model = model.to(torch.bfloat16)
    x32, b32 = spatial_model.inputs(64, device='cuda')
    args = (x32.bfloat16(), b32.bfloat16())
    compiled, report = _compile(backend, model, args, 3)
    assert report.sites == 3
    assert report.graph_count == 1 and report.graph_break_count == 0
    launches, out = _launches_per_forward(compiled, args)
    assert launches == 3  # this library's kernel ran at every site
    with torch.no_grad():
        eager16 = model(*args)
        eager32 = m32(x32, b32)
    # bf16 blocks: the compiled model is at least as close to the fp32
    # model as the bf16 eager chain is (measured 0.57 % vs 0.67 %).
    assert _rel(out, eager32) < 2e-2
    assert _rel(out, eager32) < 1.5 * _rel(eager16, eager32) + 1e-3


def test_fp32_model_matches_eager(backend):
    torch.manual_seed(1)
    model = spatial_model.SpatialNet(layers=3).cuda().eval()
    args = spatial_model.inputs(16, device='cuda', seed=1)
    compiled, report = _compile(backend, model, args, 3)
    assert report.sites == 3 and report.graph_break_count == 0
    launches, out = _launches_per_forward(compiled, args)
    assert launches == 3
    with torch.no_grad():
        ref = model(*args)
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-5)


def test_every_catalog_spelling_is_rewritten(backend):
    forms = [('divisor', 'softmax'), ('multiplier', 'softmax'),
             ('divisor', 'exp_sum'), ('multiplier', 'exp_sum')]
    torch.manual_seed(2)
    model = spatial_model.SpatialNet(layers=4, formulations=forms)
    model = model.cuda().eval()
    args = spatial_model.inputs(8, device='cuda', seed=2)
    compiled, report = _compile(backend, model, args, 4)
    assert report.sites == 4 and report.graph_break_count == 0
    assert len(report.matches) == 4  # four distinct catalog entries
    launches, out = _launches_per_forward(compiled, args)
    assert launches == 4
    with torch.no_grad():
        ref = model(*args)
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-5)


def test_compiled_model_replays_from_a_cuda_graph(backend):
    # A serving path: one compiled forward captured
    # in a CUDA graph (static input buffers, new inputs copied in, replay).
    # The operator makes no host synchronisation and no allocation the
    # caching allocator cannot serve inside the capture, so the rewritten
    # model captures and each replay runs this library's kernel per site.
    import vectra_b200  # pylint: disable=import-outside-toplevel
    torch.manual_seed(3)
    model = spatial_model.SpatialNet(layers=3).cuda().eval().bfloat16()
    args = spatial_model.inputs(32, device='cuda', dtype=torch.bfloat16,
                                seed=3)
    compiled, report = _compile(backend, model, args, 3)
    assert report.sites == 3
    static = [t.clone() for t in args]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(side):
        for _ in range(2):
            compiled(*static)  # warm the side stream
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(graph):
        static_out = compiled(*static)
    for seed in (4, 5):
        fresh = spatial_model.inputs(32, device='cuda', dtype=torch.bfloat16,
                                     seed=seed)
        for dst, src in zip(static, fresh):
            dst.copy_(src)
        before = vectra_b200.launch_count()
        graph.replay()
        torch.cuda.synchronize()
        # Replays do not pass through the host launcher, so the counter
        # does not move; the output must match a fresh compiled call.
        assert vectra_b200.launch_count() == before
        with torch.no_grad():
            want = compiled(*fresh)
        torch.testing.assert_close(static_out, want, rtol=0, atol=0)
    del graph
