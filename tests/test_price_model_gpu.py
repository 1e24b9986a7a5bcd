"""Benchmark config 5 on the reference's own price model: the compiled
PriceTransformer runs this library's kernel at every attention site.

The model, its inputs' structure, the compile pass and the export checks
are the reference's code, installed unmodified in baseline/_ref
(oracle/install_reference.py), with the one-file swap of
kernels/vectra_kernels/custom_ops.py (tests/reference_swap):

* the model: PriceTransformer(ModelConfig(embedding_dim=128,
  attribute_dim=48, d_model=256, num_heads=8, num_layers=4, ffn_dim=1024,
  num_candidates=64)) (models/price_transformer/model.py:162-244), random
  init, blocks in bfloat16 (`compile_entry.prepare`, set_block_dtype);
* compiled by `compile_entry.compile_model` (models/export/
  compile_entry.py:194-207): `compile_for_serving` with expected_sites =
  num_layers proves one graph, no graph break, every site rewritten;
* gated by `compile_entry.max_abs_error` (compile_entry.py:155-191):
  compiled vs eager at rtol 1e-3 / atol 1e-3 on seeded batches (it raises
  NumericsError otherwise), drift against the float32 eager model
  reported;
* served by the reference's `ServingModel.predict` (compile_entry.py:
  286-303) and by vectra_b200.serving with the same result bit for bit.

The model's radius trim is a torch.cond; which branch a batch takes is
recorded from the model's own predicate: BASELINE's inputs (50 km radius,
vectra_b200.workloads.price_model_inputs) take the cheap branch, the
reference's test trick (one request with a 1 m radius) the fallback.
"""

import pytest
import torch

import vectra_b200
from tests.conftest import compile_pass_installed
from vectra_b200 import serving
from vectra_b200 import workloads

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not compile_pass_installed(),
                       reason='the reference is not installed in '
                              'baseline/_ref'),
]

BATCH = 64  # the serving batch the tests compile for (the bench: 1,024)


def _config(ref, layers=4):
    return ref.model.ModelConfig(**dict(workloads.PRICE_MODEL,
                                        num_layers=layers))


def _build(ref, layers, dtype):
    torch.manual_seed(0)
    cfg = _config(ref, layers)
    spec = ref.compile_entry.ServingSpec(device='cuda', batch_size=BATCH,
                                         block_dtype=dtype)
    eager = ref.compile_entry.prepare(ref.model.PriceTransformer(cfg), spec)
    torch._dynamo.reset()  # pylint: disable=protected-access
    compiled, report, _ = ref.compile_entry.compile_model(eager, spec)
    return cfg, spec, eager, compiled, report


def _float32_twin(ref, cfg, eager):
    twin = ref.model.PriceTransformer(cfg).cuda().eval()
    twin.load_state_dict({k: v.float() for k, v in eager.state_dict().items()})
    return twin


def _cheap_branch(ref, inputs):
    """The model's own predicate for torch.cond (model.py:130-132)."""
    distance = ref.model.microhood.haversine_km(inputs[2], inputs[10])
    radius, valid = inputs[5], inputs[12]
    return bool((valid & (distance <= radius.unsqueeze(-1))).any(-1).all())


@pytest.fixture(scope='module')
def bf16_model(reference):
    return _build(reference, 4, 'bfloat16')


def test_every_site_rewritten_in_one_graph(bf16_model):
    _, _, _, _, report = bf16_model
    assert report.sites == 4
    assert report.graph_count == 1 and report.graph_break_count == 0
    assert report.matches == {'rbf_divisor_bias_softmax[half]': 4}


def test_this_librarys_kernel_runs_at_every_site(bf16_model):
    cfg, _, _, compiled, _ = bf16_model
    inputs = workloads.price_model_inputs(BATCH, seed=3, device='cuda',
                                          config=vars(cfg))
    with torch.no_grad():
        before = vectra_b200.launch_count()
        compiled(*inputs)
        torch.cuda.synchronize()
    assert vectra_b200.launch_count() - before == 4


def test_export_numerics_gate(reference, bf16_model):
    # The reference's own gate: compiled == eager (bf16 blocks) within
    # rtol 1e-3 / atol 1e-3 on seeded batches of its example inputs, and
    # the drift from the float32 eager model.
    cfg, spec, eager, compiled, _ = bf16_model
    worst, drift = reference.compile_entry.max_abs_error(
        compiled, eager, cfg, spec, batches=2,
        reference=_float32_twin(reference, cfg, eager))
    assert worst <= 1e-3 + 1e-3 * 14  # within the gate (it raises if not)
    assert drift < 0.1, drift  # bf16 blocks track the float32 model


def test_baseline_inputs_cheap_branch_matches_eager(reference, bf16_model):
    cfg, _, eager, compiled, _ = bf16_model
    for seed in (11, 12):
        inputs = workloads.price_model_inputs(BATCH, seed=seed,
                                              device='cuda',
                                              config=vars(cfg))
        assert _cheap_branch(reference, inputs)
        with torch.no_grad():
            got, want = compiled(*inputs).float(), eager(*inputs).float()
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3)


def test_fallback_branch_matches_eager(reference, bf16_model):
    cfg, _, eager, compiled, _ = bf16_model
    inputs = reference.model.example_inputs(cfg, BATCH, 'cuda', seed=21)
    radius = inputs.radius_km.clone()
    radius[3] = 1e-3  # one request with no comparable inside its radius
    inputs = inputs._replace(radius_km=radius)
    assert not _cheap_branch(reference, inputs)
    with torch.no_grad():
        got, want = compiled(*inputs).float(), eager(*inputs).float()
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3)


def test_three_layer_variant_rewrites_three_sites(reference):
    cfg, spec, eager, compiled, report = _build(reference, 3, 'bfloat16')
    assert report.sites == 3 and report.graph_break_count == 0
    reference.compile_entry.max_abs_error(compiled, eager, cfg, spec,
                                          batches=1)


def test_float32_blocks_match_eager_tightly(reference):
    cfg, _, eager, compiled, report = _build(reference, 4, 'float32')
    assert report.matches == {'rbf_divisor_bias_softmax[fp32]': 4}
    inputs = workloads.price_model_inputs(BATCH, seed=5, device='cuda',
                                          config=vars(cfg))
    with torch.no_grad():
        torch.testing.assert_close(compiled(*inputs), eager(*inputs),
                                   rtol=1e-4, atol=1e-4)


def test_serving_matches_the_reference_serving_loop(reference, bf16_model):
    # The reference's ServingModel (split, pad with the last request, run,
    # drop padding, float) and vectra_b200.serving (static slots, device
    # padding, pinned staging; no CUDA graph: the forward reads torch.cond's
    # predicate on the host) give the same values bit for bit.
    cfg, spec, _, compiled, _ = bf16_model
    ref_served = reference.compile_entry.ServingModel(compiled, cfg, spec, {})
    example = workloads.price_model_inputs(BATCH, seed=0, device='cuda',
                                           config=vars(cfg))
    ours = serving.GraphServingModel(compiled, example, capture=False)
    assert not ours.captured
    for n in (1, BATCH, BATCH + 17):
        host = workloads.price_model_inputs(n, seed=40 + n, config=vars(cfg))
        want = ref_served.predict(reference.model.PricingInputs(*host))
        got = ours.predict(host)
        assert got.shape == (n,)
        assert torch.equal(got, want)
        pinned = [t.pin_memory() for t in host]
        assert torch.equal(ours.predict(pinned), want)


def test_value_views_pass_keeps_the_outputs(reference):
    # vectra_b200.fusion hands the operator the projection's V view instead
    # of the contiguous copy the reference pass cut at. The operator reads
    # the same values either way (bit for bit, below); the compiled model,
    # whose other kernels Inductor may generate differently without the
    # copy, stays within the reference's export gate, with the same four
    # kernel launches.
    from vectra_b200 import fusion  # pylint: disable=import-outside-toplevel
    cfg, spec, eager, compiled, _ = _build(reference, 4, 'bfloat16')
    torch._dynamo.reset()  # pylint: disable=protected-access
    with fusion.installed() as p:
        fused, report, _ = reference.compile_entry.compile_model(eager, spec)
    assert report.sites == 4 and p.rewired == 4
    reference.compile_entry.max_abs_error(fused, eager, cfg, spec, batches=2)
    for seed in (31, 32):
        inputs = workloads.price_model_inputs(BATCH, seed=seed, device='cuda',
                                              config=vars(cfg))
        with torch.no_grad():
            before = vectra_b200.launch_count()
            got = fused(*inputs)
            torch.cuda.synchronize()
            assert vectra_b200.launch_count() - before == 4
            torch.testing.assert_close(got, eager(*inputs).float(),
                                       rtol=1e-3, atol=1e-3)


def test_operator_reads_a_strided_value_view_bit_for_bit():
    # The site's layout: q, k, v head-split views of one [B, N, 3 * 256]
    # projection; v as that view and as its contiguous copy.
    gen = torch.Generator(device='cuda').manual_seed(41)
    qkv = torch.randn(BATCH, 65, 3, 8, 32, device='cuda', generator=gen)
    q, k, v = qkv.bfloat16().permute(2, 0, 3, 1, 4)
    scale = torch.rand(1, 8, 1, 1, device='cuda', generator=gen) * 0.2
    bias = torch.zeros(BATCH, 1, 1, 65, device='cuda', dtype=torch.bfloat16)
    bias[::5, ..., 50:] = float('-inf')
    strided = torch.ops.vectra.rbf_attention(q, k, v, scale, bias)
    copied = torch.ops.vectra.rbf_attention(q, k, v.contiguous(), scale, bias)
    assert torch.equal(strided, copied)
