"""CUDA-graph serving of the compiled model (vectra_b200.serving) against
the reference's serving loop.

The checker is the reference's `ServingModel.predict`
(models/export/compile_entry.py:286-303), restated below: split into
chunks of `batch_size`, move to the device, pad with copies of the last
request, call the compiled model, drop the padding, float, concatenate.
Graph replay must give the same result bit for bit, for batches shorter
than, equal to and longer than the served batch, from unpinned host,
pinned host and device inputs, and this library's kernel must be inside
the captured graphs.
"""

import pytest
import torch

import vectra_b200
from tests import spatial_model
from tests.conftest import compile_pass_installed
from vectra_b200 import serving

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(
        not compile_pass_installed(),
        reason='the reference compile pass is not installed in baseline/_ref'),
]

BATCH = 48


def reference_predict(compiled, inputs, batch_size, device):
    """compile_entry.py:286-303: the reference's serving loop."""
    n = inputs[0].shape[0]
    outputs = []
    with torch.no_grad():
        for start in range(0, n, batch_size):
            chunk = [t[start:start + batch_size].to(device) for t in inputs]
            size = chunk[0].shape[0]
            if size < batch_size:
                chunk = [torch.cat([t, t[-1:].expand(batch_size - size,
                                                     *t.shape[1:])])
                         for t in chunk]
            outputs.append(compiled(*chunk)[:size].float())
    return torch.cat(outputs)


@pytest.fixture(scope='module')
def served(backend):
    torch.manual_seed(0)
    model = spatial_model.SpatialNet(layers=3).cuda().eval().bfloat16()
    example = spatial_model.inputs(BATCH, device='cuda', dtype=torch.bfloat16)
    torch._dynamo.reset()  # pylint: disable=protected-access
    compiled, report = backend.compile_for_serving(model, example,
                                                   expected_sites=3)
    assert report.sites == 3 and report.graph_break_count == 0
    before = vectra_b200.launch_count()
    gs = serving.GraphServingModel(compiled, example, slots=2, warmup=2)
    launched = vectra_b200.launch_count() - before
    return compiled, gs, launched


def test_the_operator_is_captured_in_every_slot(served):
    _, gs, launched = served
    # 2 warm-up forwards + 2 captured forwards, 3 sites each.
    assert launched == 3 * (2 + 2)
    assert gs.batch_size == BATCH
    before = vectra_b200.launch_count()
    x, b = spatial_model.inputs(BATCH, device='cuda', dtype=torch.bfloat16,
                                seed=9)
    gs.predict((x, b))
    torch.cuda.synchronize()
    # Replays do not go through the host launcher.
    assert vectra_b200.launch_count() == before


@pytest.mark.parametrize('n', [1, 17, BATCH, BATCH + 1, 3 * BATCH + 5])
@pytest.mark.parametrize('where', ['host', 'pinned', 'device'])
def test_matches_the_reference_serving_loop(served, n, where):
    compiled, gs, _ = served
    x, b = spatial_model.inputs(n, dtype=torch.bfloat16, seed=n)
    if where == 'pinned':
        x, b = x.pin_memory(), b.pin_memory()
    elif where == 'device':
        x, b = x.cuda(), b.cuda()
    got = gs.predict((x, b))
    want = reference_predict(compiled, (x, b), BATCH, 'cuda')
    assert got.dtype == torch.float32 and got.shape == (n,)
    assert got.device == want.device
    assert torch.equal(got, want)


def test_mixed_host_and_device_inputs(served):
    compiled, gs, _ = served
    x, b = spatial_model.inputs(2 * BATCH + 3, dtype=torch.bfloat16, seed=21)
    got = gs.predict((x, b.cuda()))
    want = reference_predict(compiled, (x, b), BATCH, 'cuda')
    assert torch.equal(got, want)


def test_back_to_back_calls_reuse_slots_safely(served):
    # Many chunks through two slots, then new inputs: no chunk may see
    # another call's rows.
    compiled, gs, _ = served
    outs, wants = [], []
    for seed in range(4):
        x, b = spatial_model.inputs(5 * BATCH - seed, dtype=torch.bfloat16,
                                    seed=100 + seed)
        x = x.pin_memory()
        outs.append(gs.predict((x, b)))
        wants.append(reference_predict(compiled, (x, b), BATCH, 'cuda'))
    for got, want in zip(outs, wants):
        assert torch.equal(got, want)


def test_rejects_inputs_of_another_shape_or_dtype(served):
    _, gs, _ = served
    x, b = spatial_model.inputs(4, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        gs.predict((x[..., :-1], b))
    with pytest.raises(ValueError):
        gs.predict((x.float(), b))
    with pytest.raises(ValueError):
        gs.predict((x,))
    with pytest.raises(ValueError):
        gs.predict((x[:0], b[:0]))
