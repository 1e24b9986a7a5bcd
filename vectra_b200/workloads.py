"""Seeded synthetic inputs for the benchmark configurations, and their
algorithmic byte / FLOP counts (the roofline numerators).

The reference measures on generated data too (kernels/benchmarks/
throughput.py:97-111 `problem`); these generators follow the benchmark
configuration descriptions instead, with fixed seeds:

1. CPU-scale serving: B=8, H=4, Lq=1, Lk=16, D=32, fp32; q,k,v ~ N(0,1);
   gamma_h ~ U(0.05, 0.5); no mask.
2. Serving: B=1024, H=8, Lq=1, Lk=64, D=64, bf16; q,k,v ~ N(0,1)/sqrt(D);
   gamma_h ~ U(0.1, 1.0); dense.
3. Variable comparable counts: B=4096, H=8, Lq=1, Lk_max=128, D=64, bf16;
   valid length ~ U{8..128} as a 0/-inf bf16 key_bias [B,1,1,128] built
   like the model's (models/price_transformer/model.py:233-236); keys are
   cluster centres N(0,1) (8 per plane) plus N(0, 0.1) jitter; q ~ N(0,1);
   v ~ N(0,1)/sqrt(D); gamma_h ~ U(0.1, 2.0).
4. Long sequences: B=16, H=16, Lq=Lk=4096, D=128, bf16;
   q,k,v ~ N(0,1)/sqrt(D); gamma_h ~ U(0.01, 0.2); no mask.
5. One attention site of the compiled price model (benchmark config 5:
   batch 1024 targets, 64 comparables, d_model 256, 8 heads of D=32, bf16):
   q, k, v are head-transposed views of one [B, N=65, 3, H, D] projection
   (row stride 3*H*D, the layout the compile pass hands the operator),
   projection values ~ N(0,1)/sqrt(D); the coefficient 1/(2 sigma_h^2) with
   log sigma_h ~ N(0.7, 0.3); a [B,1,1,N] bf16 key bias of zeros (every
   comparable valid).

`price_model_inputs` builds the whole price model's inputs for benchmark
config 5 (the reference's `PricingInputs`, models/price_transformer/
model.py:58-88, in forward-argument order): targets and comparables placed
uniformly over a 50 km box, comparables' log sale prices ~ N(13, 0.6^2)
(lognormal prices), standardised attributes ~ N(0, 1), embeddings
tanh(N(0, 1)) as the reference's `example_inputs` draws them
(model.py:252-282), sale days up to a few years before the valuation day,
GeoHash-6 cells of the locations, every comparable valid, and a 50 km
search radius, so every request has comparables inside its radius and the
model's radius trim takes its cheap branch.
"""

import dataclasses
import math

import torch

DTYPES = {'f32': torch.float32, 'f16': torch.float16, 'bf16': torch.bfloat16}

SHAPES = {  # B, H, Nq, Nk, D, dtype
    1: (8, 4, 1, 16, 32, 'f32'),
    2: (1024, 8, 1, 64, 64, 'bf16'),
    3: (4096, 8, 1, 128, 64, 'bf16'),
    4: (16, 16, 4096, 4096, 128, 'bf16'),
    5: (1024, 8, 65, 65, 32, 'bf16'),
}
NAMES = {
    1: 'config1 B=8 H=4 Lq=1 Lk=16 D=32 fp32',
    2: 'serving B=1024 H=8 Lq=1 Lk=64 D=64 bf16',
    3: 'variable-count B=4096 H=8 Lq=1 Lk_max=128 D=64 bf16 padding bias',
    4: 'long B=16 H=16 Lq=Lk=4096 D=128 bf16',
    5: 'compiled-model attention site B=1024 N=65 H=8 D=32 bf16 strided',
}


@dataclasses.dataclass
class Workload:
    config: int
    dtype: str
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    scale: torch.Tensor
    key_bias: torch.Tensor | None
    lengths: torch.Tensor | None  # valid keys per batch row (config 3)

    @property
    def batch(self) -> int:
        return self.q.shape[0]

    def tensors(self):
        return self.q, self.k, self.v, self.scale, self.key_bias

    def slice(self, lo: int, hi: int) -> 'Workload':
        """Batch rows [lo, hi); the scale is per head and is shared."""
        return Workload(
            self.config, self.dtype, self.q[lo:hi], self.k[lo:hi],
            self.v[lo:hi], self.scale,
            None if self.key_bias is None else self.key_bias[lo:hi],
            None if self.lengths is None else self.lengths[lo:hi])


def make(config: int, device='cuda', seed: int = 0,
         batch: int | None = None) -> Workload:
    """Builds config `config` (1-4) on `device` from `seed`.

    `batch` overrides the batch size (tests use it for cheap slices); the
    values of row b do not depend on the batch size only for config 1
    (generation is whole-tensor).
    """
    B, H, nq, nk, D, dtype = SHAPES[config]
    if batch is not None:
        B = batch
    td = DTYPES[dtype]
    gen = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=gen, device=device)

    def rand(*shape):
        return torch.rand(*shape, generator=gen, device=device)

    lengths = bias = None
    if config == 1:
        q, k, v = randn(B, H, nq, D), randn(B, H, nk, D), randn(B, H, nk, D)
        scale = 0.05 + 0.45 * rand(1, H, 1, 1)
    elif config in (2, 4):
        inv = 1.0 / math.sqrt(D)
        q = randn(B, H, nq, D) * inv
        k = randn(B, H, nk, D) * inv
        v = randn(B, H, nk, D) * inv
        scale = (0.1 + 0.9 * rand(1, H, 1, 1) if config == 2
                 else 0.01 + 0.19 * rand(1, H, 1, 1))
    elif config == 3:
        q = randn(B, H, nq, D)
        centres = randn(B, H, 8, D)
        assign = torch.randint(0, 8, (B, H, nk), generator=gen,
                               device=device)
        k = torch.gather(centres, 2, assign[..., None].expand(B, H, nk, D))
        k = k + 0.1 * randn(B, H, nk, D)
        v = randn(B, H, nk, D) / math.sqrt(D)
        scale = 0.1 + 1.9 * rand(1, H, 1, 1)
        lengths = torch.randint(8, nk + 1, (B,), generator=gen,
                                device=device)
        valid = torch.arange(nk, device=device)[None, :] < lengths[:, None]
        bias = torch.zeros(B, nk, device=device).masked_fill(
            ~valid, float('-inf')).to(td)[:, None, None, :]
    elif config == 5:
        qkv = randn(B, nq, 3, H, D) / math.sqrt(D)
        q, k, v = qkv.to(td).permute(2, 0, 3, 1, 4)
        sigma = torch.exp(0.7 + 0.3 * randn(1, H, 1, 1))
        scale = 1.0 / (2.0 * sigma * sigma)
        bias = torch.zeros(B, 1, 1, nk, device=device, dtype=td)
        return Workload(config, dtype, q, k, v, scale, bias, None)
    else:
        raise ValueError(f'unknown config {config}')
    return Workload(config, dtype, q.to(td), k.to(td), v.to(td), scale,
                    bias, lengths)


def algorithmic_bytes(w: Workload) -> int:
    """HBM bytes one pass must move: Q, the K/V rows that carry weight,
    O, the scale and the bias (each read or written once).

    Keys masked by a -inf bias contribute nothing and are not counted
    (config 3); without a bias every key counts.
    """
    B, H, nq, D = w.q.shape
    nk, dv = w.k.shape[2], w.v.shape[3]
    es = w.q.element_size()
    qo = B * H * nq * (D + dv) * es
    if w.lengths is not None:
        keys = int(w.lengths.sum().item())
    else:
        keys = B * nk
    kv = keys * H * (D + dv) * es
    extra = w.scale.numel() * w.scale.element_size()
    if w.key_bias is not None:
        extra += w.key_bias.numel() * w.key_bias.element_size()
    return qo + kv + extra


def dense_bytes(w: Workload) -> int:
    """Bytes if every key row were read (what the reference kernel reads)."""
    B, H, nq, D = w.q.shape
    nk, dv = w.k.shape[2], w.v.shape[3]
    es = w.q.element_size()
    extra = w.scale.numel() * w.scale.element_size()
    if w.key_bias is not None:
        extra += w.key_bias.numel() * w.key_bias.element_size()
    return B * H * (nq * (D + dv) + nk * (D + dv)) * es + extra


def algorithmic_flops(w: Workload) -> int:
    """The two contractions, 2*Nq*Nk*(D + Dv) per plane (exponentials and
    norms excluded, the FlashAttention convention)."""
    B, H, nq, D = w.q.shape
    nk, dv = w.k.shape[2], w.v.shape[3]
    return 2 * B * H * nq * nk * (D + dv)


# Benchmark config 5: the price model's serving shape.
PRICE_MODEL = dict(embedding_dim=128, attribute_dim=48, d_model=256,
                   num_heads=8, num_layers=4, ffn_dim=1024, num_candidates=64)
PRICE_BATCH = 1024
PRICE_RADIUS_KM = 50.0
_BOX_CENTRE = (37.7749, -122.4194)  # degrees (latitude, longitude)
_BOX_KM = 50.0
_KM_PER_DEGREE = 6371.0088 * math.pi / 180.0


def geohash_cells(lat: torch.Tensor, lng: torch.Tensor,
                  precision: int = 6) -> torch.Tensor:
    """GeoHash cells as integers (int64): 5 * precision bits, longitude and
    latitude bisection bits interleaved, longitude first, most significant
    bit first (the GeoHash definition; data/geo.py:107 in the reference).
    A coordinate's index on an axis with n bits is floor((x - lo) /
    (hi - lo) * 2^n), the result of n bisections."""
    lng_bits = (5 * precision + 1) // 2
    lat_bits = 5 * precision // 2

    def index(x, lo, hi, bits):
        scaled = ((x.double() - lo) / (hi - lo) * (1 << bits)).floor()
        return scaled.clamp(0, (1 << bits) - 1).long()

    col = index(lng, -180.0, 180.0, lng_bits)
    row = index(lat, -90.0, 90.0, lat_bits)
    cell = torch.zeros_like(col)
    for i in range(5 * precision):
        if i % 2 == 0:
            lng_bits -= 1
            bit = (col >> lng_bits) & 1
        else:
            lat_bits -= 1
            bit = (row >> lat_bits) & 1
        cell = (cell << 1) | bit
    return cell


def price_model_inputs(batch: int = PRICE_BATCH, seed: int = 0,
                       device='cpu', config=None):
    """Benchmark config 5's inputs for the price model: 13 tensors in the
    forward's argument order (query_embedding, query_attributes,
    query_location, query_cell6, valuation_day, radius_km, cand_embedding,
    cand_attributes, cand_log_price, cand_sale_day, cand_location,
    cand_cell6, cand_valid). Generated on the CPU from `seed`, then moved to
    `device`."""
    cfg = dict(PRICE_MODEL if config is None else config)
    e, a, k = cfg['embedding_dim'], cfg['attribute_dim'], \
        cfg['num_candidates']
    gen = torch.Generator().manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=gen)

    def rand(*shape):
        return torch.rand(*shape, generator=gen)

    half_lat = 0.5 * _BOX_KM / _KM_PER_DEGREE
    half_lng = half_lat / math.cos(math.radians(_BOX_CENTRE[0]))

    def locations(*shape):
        lat = _BOX_CENTRE[0] + half_lat * (2 * rand(*shape) - 1)
        lng = _BOX_CENTRE[1] + half_lng * (2 * rand(*shape) - 1)
        return torch.stack([lat, lng], dim=-1)

    query_location = locations(batch)
    cand_location = locations(batch, k)
    tensors = (
        torch.tanh(randn(batch, e)),
        randn(batch, a),
        query_location,
        geohash_cells(query_location[..., 0], query_location[..., 1]),
        torch.full((batch,), 20000.0),
        torch.full((batch,), PRICE_RADIUS_KM),
        torch.tanh(randn(batch, k, e)),
        randn(batch, k, a),
        13.0 + 0.6 * randn(batch, k),
        20000.0 - 900.0 * randn(batch, k).abs(),
        cand_location,
        geohash_cells(cand_location[..., 0], cand_location[..., 1]),
        torch.ones(batch, k, dtype=torch.bool),
    )
    return tuple(t.to(device) for t in tensors)
