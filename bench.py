"""Benchmark of torch.ops.vectra.rbf_attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--impl vectra|reference] [--scaling strong|weak]

One step is one pass of the operator over one batch of the workload
(default: benchmark config 2, the serving shape B=1024, H=8, Lq=1, Lk=64,
D=64, bf16). With N GPUs (torchrun, one process per GPU) the batch is
sharded (strong scaling, the default): every rank generates the same seeded
batch and keeps its contiguous slice (vectra_b200.sharding.shard_range), so
the ranks together do the one-GPU job; there is no collective on the data
path. The value is the batch's queries divided by the slowest rank's device
time. `--scaling weak` gives every rank its own batch of the configured
size instead; with N > 1 the strong line also carries the weak figure
(`extra.weak`).

Rank 0 prints one JSON line with:
* value: queries/s (or TFLOP/s for config 4), inputs resident in HBM,
  CUDA events over exactly K steps bracketed by barrier + synchronize,
  max over ranks;
* e2e: the same metric through the public API with pinned host buffers,
  host->device input copies and the device->host output copy of every step
  inside the timed region (steps pipelined over a copy and a compute
  stream);
* roofline: the kernel's algorithmic bytes (or FLOPs) per launch over its
  event-timed launch duration, against MEASURED_PEAKS.json;
* cpu_baseline: the oracle's port of the reference operator's CPU
  implementation (reference.matmul_rbf_attention, the default impl of
  vectra::rbf_attention) timed on this host's cores on a bounded sample
  (rank 0, N == 1 only);
* extra.long_sequence (config 2, N == 1): benchmark config 4 (B=16, H=16,
  L=4096, D=128) through the tensor-core kernel, TFLOP/s by CUDA events;
* extra.reference_triton_kernel (N == 1): the reference's own Triton kernel
  on the same inputs and GPU, timed the same way, for context;
* clocks: nvidia-smi samples taken while the GPU ran the kernel.

`--impl reference` times the reference's CPU implementation of the path
(the operator's default impl, kernels/vectra_kernels/custom_ops.py:52-72 ->
reference.matmul_rbf_attention, reference.py:79-99, through the oracle's
NumPy port: the reference is Python and ships no compiled CPU code; the
port is also ~2.6x faster here than the port of the eager chain) with all
host threads on bounded samples of the same workload. It never loads this
library: the seeded generators are read from vectra_b200/workloads.py by
path, and its `config` is the GPU line's, key for key.
"""

import argparse
import concurrent.futures
import importlib.util
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=2000)
    p.add_argument('--warmup', type=int, default=20)
    p.add_argument('--config', type=int, default=2,
                   choices=(1, 2, 3, 4, 5))
    p.add_argument('--impl', default='vectra', choices=('vectra',
                                                         'reference'))
    p.add_argument('--e2e-steps', type=int, default=20)
    p.add_argument('--scaling', default='strong', choices=('strong', 'weak'),
                   help='strong: the GPUs split one configured batch; weak: '
                        'each GPU runs the configured batch')
    p.add_argument('--graph-calls', type=int, default=0,
                   help='operator calls per replayed CUDA graph in the timed '
                        'region (0: a multiple of the input sets, >= 12)')
    p.add_argument('--cpu-seconds', type=float, default=10.0)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-extra', action='store_true',
                   help='skip the extra measurements (weak scaling at N > 1, '
                        'config 4 at N == 1)')
    p.add_argument('--kernel', default='auto',
                   choices=('auto', 'decode', 'tc', 'small', 'small_tc',
                            'generic'),
                   help='operator runs: pin the kernel (default: the one the '
                        'library selects), e.g. to time or profile the '
                        'tcgen05 form of the small kernel on config 5')
    p.add_argument('--shard-of', type=int, default=1, metavar='N',
                   help='one GPU only: time the shard that one rank of an '
                        'N-GPU strong-scaling run gets (the per-GPU work '
                        'of that run), e.g. for the small-shard launch '
                        'list')
    p.add_argument('--profile', action='store_true',
                   help='warm-up and K steps only (for ncu): no clock soak, '
                        'no e2e, no CPU baseline, no JSON line')
    p.add_argument('--model', action='store_true',
                   help='config 5 only: the reference price model compiled '
                        'whole (predictions/s) instead of one site')
    p.add_argument('--scan', choices=('l2', 'pq'),
                   help='the index-shard scan path instead of the operator: '
                        'exhaustive L2 or PQ top-k (queries/s)')
    args = p.parse_args(argv)
    if args.model and args.config != 5:
        p.error('--model needs --config 5')
    if args.scan and args.model:
        p.error('--scan and --model are separate workloads')
    if args.shard_of < 1:
        p.error('--shard-of needs N >= 1')
    if (args.shard_of > 1 or args.kernel != 'auto') and (args.scan or
                                                         args.model):
        p.error('--shard-of and --kernel apply to the operator runs only')
    return args


# ---------------------------------------------------------------------------
# Shared descriptions
# ---------------------------------------------------------------------------

def workloads_module():
    """vectra_b200/workloads.py, loaded from its file (torch only): the
    reference arm and the CPU baseline use the seeded generators without
    importing the package, whose import loads this library's kernels."""
    name = 'vectra_bench_workloads'
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            name, os.path.join(ROOT, 'vectra_b200', 'workloads.py'))
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
    return sys.modules[name]


def metric_for(config, model=False):
    if model:
        return ('price-model predictions/s, compiled PriceTransformer with '
                'every RBF site rewritten (B=1024 targets x 65 tokens, '
                'd_model 256, 4 layers, H=8 D=32, bf16 blocks)',
                'predictions/s')
    if config == 5:
        return ('RBF-attn compiled-model site targets/s (B=1024 N=65 H=8 '
                'D=32 bf16, strided q/k/v)', 'targets/s')
    if config == 4:
        return ('RBF-attn TFLOP/s, long sequences (B=16 H=16 L=4096 D=128 '
                'bf16)', 'TFLOP/s')
    return ('RBF-attn queries/s @B=1024 + achieved HBM GB/s vs 8 TB/s, '
            '1/2/4/8 B200', 'queries/s')


def plan(config, scaling, world):
    """Batch sizes and input rotation of a run, from the shapes alone (both
    arms report them): the largest per-GPU batch, the job's batch, one
    input set's bytes on a GPU, and how many sets rotate so the timed calls
    read more than L2 holds."""
    w = workloads_module()
    b, h, nq, nk, d, dt = w.SHAPES[config]
    es = 4 if dt == 'f32' else 2
    strong = scaling == 'strong'
    per_gpu = -(-b // world) if strong else b
    bias = nk * 2 if config in (3, 5) else 0  # a bf16 bias row per batch row
    set_bytes = per_gpu * (h * (nq + nk) * 2 * d * es + bias) + h * 4
    n_sets = max(1, min(32 if strong else 8, -(-3 * L2_BYTES // set_bytes)))
    return {'per_gpu': per_gpu, 'global_batch': b if strong else b * world,
            'set_bytes': set_bytes, 'n_sets': n_sets}


def line_config(args, world):
    """The JSON line's `config`, the same in both arms."""
    w = workloads_module()
    p = plan(args.config, args.scaling, world)
    total = p['n_sets'] * p['set_bytes']
    return {
        'workload': w.NAMES[args.config],
        'queries_per_gpu': p['per_gpu'],
        'global_batch': p['global_batch'],
        'parallelism': f'batch-sharded x{world} ({args.scaling} scaling), '
                       'no collective',
        'l2': f'{p["n_sets"]} rotating input sets of '
              f'{p["set_bytes"] / 1e6:.1f} MB per GPU '
              f'({total / 2**20:.0f} MiB in all; L2 {L2_BYTES >> 20} MiB)',
    }


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path, encoding='utf-8') as f:
            d = json.load(f)
        return d['hbm_gbs'], d['bf16_tflops'], 'measured'
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 'fallback'


def ncu_traffic(config, name=None, key='dram_bytes_per_launch_full',
                kernel=None):
    """DRAM bytes per launch from the committed ncu summary, if any
    (profiles/rbf_<kernel>_config<config>.txt for the kernel the library
    selects, or the pinned `kernel`; or profiles/<name>.txt)."""
    if name is None:
        if kernel in (None, 'auto'):
            kernel = {4: 'tc', 5: 'small'}.get(config, 'decode')
        name = f'rbf_{kernel}_config{config}'
    path = os.path.join(ROOT, 'profiles', f'{name}.txt')
    try:
        with open(path, encoding='utf-8') as f:
            for line in f:
                m = re.match(re.escape(key) + r':\s*([0-9.eE+]+)',
                             line.strip())
                if m:
                    return float(m.group(1))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# CPU side: the reference formulation through the oracle port.
# ---------------------------------------------------------------------------

def cpu_sample(config, n_queries, seed=1):
    """A bounded host-side sample of the workload (same generator rules)."""
    w = workloads_module().make(config, device='cpu', seed=seed,
                                batch=n_queries if config != 4 else 1)
    tensors = [None if t is None else t.float().numpy() for t in w.tensors()]
    return w, tensors


def cpu_model():
    """The host CPU's model name (Linux), for the CPU baseline's record."""
    try:
        with open('/proc/cpuinfo', encoding='utf-8') as f:
            for line in f:
                if line.startswith('model name'):
                    return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


class CpuRunner:
    """The oracle's port of the operator's CPU implementation (formulation
    'matmul', reference.matmul_rbf_attention, the default impl of
    vectra::rbf_attention) or of the eager chain ('eager',
    reference.eager_rbf_attention, north_star's CPU path) on `threads` host
    threads over a fixed sample of the workload, prepared once; run(seconds)
    times whole passes over it for about `seconds` (at least one pass)."""

    def __init__(self, config, threads, formulation='matmul'):
        sys.path.insert(0, ROOT)
        from oracle import rbf_oracle  # pylint: disable=import-outside-toplevel
        self.config = config
        fn = (rbf_oracle.eager_rbf_attention if formulation == 'eager'
              else rbf_oracle.matmul_rbf_attention)
        what = ('eager-chain port' if formulation == 'eager'
                else 'matmul port (the op CPU impl)')
        if config == 4:
            # One (b, h) plane slice: 64 query rows against all 4096 keys.
            _, (q, k, v, sc, _b) = cpu_sample(4, 1)
            q, k, v, sc = q[:, :1, :64], k[:, :1], v[:, :1], sc[:, :1]
            self.work_items = [None]
            self.pool = None
            self.per_pass = 2 * 64 * 4096 * (128 + 128) / 1e12
            self.unit, self.cores = 'TFLOP/s', 1
            self.sample = f'{what}, 1 plane x 64 queries x 4096 keys'
            self._pass = lambda: fn(q, k, v, sc)
            return
        n = {1: 8, 5: 32}.get(config, 256)
        _, (q, k, v, sc, b) = cpu_sample(config, n)
        chunks = [c for c in np.array_split(np.arange(n), threads) if len(c)]
        parts = [rbf_oracle.sample_planes(q, k, v, sc, b, c) for c in chunks]
        self.pool = concurrent.futures.ThreadPoolExecutor(len(parts))
        self.per_pass = n
        self.unit, self.cores = metric_for(config)[1], len(parts)
        self.sample = f'{what}, {n} batch rows per pass'
        self._pass = lambda: list(self.pool.map(lambda a: fn(*a), parts))

    def run(self, seconds):
        t0 = time.perf_counter()
        n = 0
        while n == 0 or time.perf_counter() - t0 < seconds:
            self._pass()
            n += 1
        return n * self.per_pass / (time.perf_counter() - t0)

    def close(self):
        if self.pool is not None:
            self.pool.shutdown()


def time_cpu(config, seconds, threads, formulation='matmul'):
    """One timing of CpuRunner: (value, unit, cores, sample)."""
    runner = CpuRunner(config, threads, formulation)
    try:
        runner.run(min(seconds, 1.0) / 4)  # warm-up
        value = runner.run(seconds)
    finally:
        runner.close()
    return value, runner.unit, runner.cores, runner.sample


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    if rank != 0:
        return 0
    metric, unit = metric_for(args.config)
    threads = os.cpu_count() or 1
    # About two minutes in all, whatever K and W are (at least 20 ms of
    # CPU work per step).
    per_step = max(0.02, min(5.0, 120.0 / max(1, args.steps + args.warmup)))
    runner = CpuRunner(args.config, threads)
    try:
        for _ in range(args.warmup):
            runner.run(per_step / 4)
        vals = [runner.run(per_step) for _ in range(args.steps)]
    finally:
        runner.close()
    cores, sample = runner.cores, runner.sample
    value = float(statistics.median(vals))
    line = {
        'impl': 'reference', 'metric': metric, 'value': value, 'unit': unit,
        'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': True, 'scaling': args.scaling,
        'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded; benchmark config shapes and '
                'distributions)',
        'config': line_config(args, world),
        'cpu_baseline': {'value': value, 'unit': unit, 'cores': cores,
                         'kind': 'port', 'sample': sample,
                         'cpu_model': cpu_model(), 'device': 'host CPU'},
        'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    }
    emit(line)
    return 0


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clock, throttle-reason and utilisation samples every
    100 ms."""

    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,'
             'clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,'
             'clocks_event_reasons.sw_power_cap,utilization.gpu')

    def __init__(self, device_index):
        self.proc = None
        self.device = device_index
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--id={device_index}',
                 f'--query-gpu={self.QUERY}', '--format=csv,noheader,nounits',
                 '-lms', '100'], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [],
                    'samples': 0, 'util_max_pct': None}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(',') for r in out.strip().splitlines() if r.strip()]
        sm, smax, reasons, util = [], None, set(), []
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown',
                 'sw_power_cap']
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for name, flag in zip(names, r[5:9]):
                    if flag.strip().lower() == 'active':
                        reasons.add(name)
                util.append(float(r[9]))
            except (ValueError, IndexError):
                continue
        loaded = [x for x in sm if smax and x > 0.5 * smax] or sm
        return {'sm_mhz': statistics.median(loaded) if loaded else None,
                'sm_max_mhz': smax, 'reasons': sorted(reasons),
                'samples': len(sm), 'util_max_pct': max(util) if util else None}


class Gpu:
    """The rank's device, process group and timing helpers."""

    def __init__(self, timeout_s=300):
        import datetime  # pylint: disable=import-outside-toplevel
        import torch  # pylint: disable=import-outside-toplevel
        import torch.distributed as dist  # pylint: disable=import-outside-toplevel
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get('WORLD_SIZE', '1'))
        self.rank = int(os.environ.get('RANK', '0'))
        self.local = int(os.environ.get('LOCAL_RANK', '0'))
        torch.cuda.set_device(self.local)
        self.dev = torch.device('cuda', self.local)
        self.distributed = self.world > 1
        if self.distributed:
            dist.init_process_group(
                'nccl', device_id=self.dev,
                timeout=datetime.timedelta(seconds=timeout_s))

    def barrier(self):
        if self.distributed:
            self.dist.barrier(device_ids=[self.local])
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x):
        from vectra_b200 import sharding  # pylint: disable=import-outside-toplevel
        return sharding.max_over_ranks(x, device=self.dev)

    def sum_over_ranks(self, x):
        if not self.distributed:
            return float(x)
        t = self.torch.tensor([float(x)], dtype=self.torch.float64,
                              device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def busy_gpus(self, clocks):
        """How many ranks' GPUs nvidia-smi saw busy (utilisation above 0)
        while the rank's sampler ran (the soak and the timed region)."""
        util = clocks.get('util_max_pct')
        return int(round(self.sum_over_ranks(1.0 if util and util > 0 else 0.0)))

    def close(self):
        if self.distributed:
            self.dist.destroy_process_group()


def graph_timed(gpu, step, n_sets, steps, graph_calls=0):
    """Times exactly `steps` calls of step(i) (call i on input set i mod
    n_sets) replayed from CUDA graphs that hold G consecutive calls (G = the
    smallest multiple of n_sets that is at least 12, or `graph_calls`), so
    the host's per-call dispatch never starves the GPU; a second graph holds
    the calls left over. Returns (device ms of the region, this library's
    launches in it, G)."""
    import vectra_b200  # pylint: disable=import-outside-toplevel
    torch = gpu.torch
    stream = torch.cuda.current_stream(gpu.dev)
    per_graph = graph_calls or n_sets * -(-12 // n_sets)
    per_graph = max(1, min(per_graph, steps))
    full, rest = divmod(steps, per_graph)
    capture_stream = torch.cuda.Stream(gpu.dev)
    capture_stream.wait_stream(stream)

    def capture(n_calls):
        g = torch.cuda.CUDAGraph()
        before = vectra_b200.launch_count()
        with torch.cuda.graph(g, stream=capture_stream):
            for c in range(n_calls):
                step(c)
        return g, vectra_b200.launch_count() - before

    with torch.cuda.stream(capture_stream):
        for i in range(n_sets):
            step(i)  # warm the capture stream
        capture_stream.synchronize()
        main_graph, main_launches = capture(per_graph)
        rest_graph, rest_launches = capture(rest) if rest else (None, 0)
    stream.wait_stream(capture_stream)
    main_graph.replay()
    if rest_graph is not None:
        rest_graph.replay()
    region0 = torch.cuda.Event(enable_timing=True)
    region1 = torch.cuda.Event(enable_timing=True)
    gpu.barrier()
    region0.record(stream)
    for _ in range(full):
        main_graph.replay()
    if rest_graph is not None:
        rest_graph.replay()
    region1.record(stream)
    torch.cuda.synchronize()
    gpu.barrier()
    launches = full * main_launches + rest_launches
    region_ms = region0.elapsed_time(region1)
    del main_graph, rest_graph
    return region_ms, launches, per_graph


def long_sequence_extra(gpu, calls=20):
    """Benchmark config 4 through the operator (the tensor-core kernel),
    CUDA events over `calls` back-to-back calls on two input sets of 1 GB
    each (> L2): TFLOP/s and the fraction of the measured bf16 peak."""
    import vectra_b200  # pylint: disable=import-outside-toplevel
    from vectra_b200 import workloads  # pylint: disable=import-outside-toplevel
    torch = gpu.torch
    sets = [workloads.make(4, device=gpu.dev, seed=s) for s in range(2)]
    op = torch.ops.vectra.rbf_attention
    for i in range(3):
        op(*sets[i % 2].tensors())
    stream = torch.cuda.current_stream(gpu.dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    before = vectra_b200.launch_count()
    e0.record(stream)
    for i in range(calls):
        op(*sets[i % 2].tensors())
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / calls
    flops = workloads.algorithmic_flops(sets[0])
    _, tflops_peak, kind = peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    out = {'workload': workloads.NAMES[4],
           'kernel': vectra_b200.kernel_for(*sets[0].tensors()),
           'ms_per_call': ms, 'value': tflops, 'unit': 'TFLOP/s',
           'calls': calls, 'launches': vectra_b200.launch_count() - before,
           'frac_of_bf16_peak': tflops / tflops_peak,
           'peak': tflops_peak, 'peak_kind': f'bf16 dense, {kind} (burst)'}
    del sets
    torch.cuda.empty_cache()
    return out


def reference_triton_extra(gpu, sets, calls=240):
    """The reference's own GPU kernel on the same input sets, for context:
    its launcher `rbf_attention_forward` (kernels/vectra_kernels/
    spatial_rbf_attention.py:177-281, the Triton kernel the operator's CUDA
    registration called, custom_ops.py:75-85), JIT-compiled by this image's
    Triton for the B200, imported from the reference's unmodified install
    in baseline/_ref (its module registers no operator). Calls replayed
    from a CUDA graph and timed with CUDA events, like this library's.
    None when the install or Triton is missing."""
    ref = os.path.join(ROOT, 'baseline', '_ref')
    if not os.path.isfile(os.path.join(ref, 'INSTALL.json')):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    try:
        from vectra_kernels import spatial_rbf_attention  # pylint: disable=import-outside-toplevel
    except ImportError as exc:
        return {'unavailable': f'cannot import the reference kernel: {exc}'}
    torch = gpu.torch
    n = len(sets)

    def step(i):
        w = sets[i % n]
        return spatial_rbf_attention.rbf_attention_forward(
            w.q, w.k, w.v, w.scale, w.key_bias)

    for i in range(max(3, n)):
        step(i)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(gpu.dev)
    side.wait_stream(torch.cuda.current_stream(gpu.dev))
    per_graph = n * -(-12 // n)
    with torch.cuda.stream(side):
        for i in range(n):
            step(i)
        side.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for c in range(per_graph):
                step(c)
    stream = torch.cuda.current_stream(gpu.dev)
    stream.wait_stream(side)
    graph.replay()
    reps = max(1, calls // per_graph)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del graph
    ms = e0.elapsed_time(e1) / (reps * per_graph)
    return {'kernel': 'reference Triton kernel (spatial_rbf_attention.'
                      'rbf_attention_forward), JIT-compiled for sm_100',
            'ms_per_call': ms, 'calls': reps * per_graph}


def run_vectra(args):
    sys.path.insert(0, ROOT)
    gpu = Gpu()
    torch = gpu.torch
    import vectra_b200  # pylint: disable=import-outside-toplevel
    from vectra_b200 import sharding  # pylint: disable=import-outside-toplevel
    from vectra_b200 import workloads  # pylint: disable=import-outside-toplevel
    world, rank, dev = gpu.world, gpu.rank, gpu.dev
    # --shard-of N on one GPU: this GPU plays rank 0 of N (strong scaling).
    shards = args.shard_of if world == 1 else world

    def make_set(i, scaling):
        """Input set i on this rank: its shard of the identically seeded
        batch (strong) or its own batch (weak)."""
        if scaling == 'weak':
            return workloads.make(args.config, device=dev,
                                  seed=1000 * rank + i)
        full = workloads.make(args.config, device=dev, seed=i)
        lo, hi = sharding.shard_range(full.batch, shards, rank)
        part = full.slice(lo, hi)
        return workloads.Workload(
            part.config, part.dtype,
            *(None if t is None else t.clone()
              for t in (part.q, part.k, part.v, part.scale, part.key_bias,
                        part.lengths)))

    p = plan(args.config, args.scaling, shards)
    n_sets = p['n_sets']
    sets = [make_set(i, args.scaling) for i in range(n_sets)]
    w0 = sets[0]
    if shards != world:
        # The job is the shard: its queries, not the configured batch.
        p['global_batch'] = w0.batch
    alg_bytes = workloads.algorithmic_bytes(w0)
    flops = workloads.algorithmic_flops(w0)
    if args.kernel == 'auto':
        op = torch.ops.vectra.rbf_attention
    else:
        # The same operator with the kernel pinned (--kernel).
        vectra_b200.kernel_for(*w0.tensors(), kernel=args.kernel)

        def op(*a):
            return vectra_b200.rbf_attention_with_kernel(
                *a, kernel=args.kernel)

    def step(i):
        w = sets[i % n_sets]
        return op(w.q, w.k, w.v, w.scale, w.key_bias)

    # Warm-up (also loads the module and sets kernel attributes), then a
    # short soak so the clock sampler sees the GPU under this load (the
    # sampler keeps running through the timed region).
    for i in range(max(3, args.warmup)):
        step(i)
    if args.profile:
        # One NVTX range per operator call, named as the reference's
        # benchmarks name theirs (kernels/benchmarks/bandwidth.py:74-77),
        # so ncu --nvtx --nvtx-include vectra_region/ selects the same work.
        for i in range(args.steps):
            torch.cuda.nvtx.range_push('vectra_region')
            step(i)
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        gpu.close()
        return 0
    sampler = ClockSampler(gpu.local)
    torch.cuda.synchronize()
    t_soak = time.perf_counter()
    i = 0
    while time.perf_counter() - t_soak < 0.6:
        step(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize()

    # Timed region: exactly K steps, one operator call on one batch (shard)
    # each, replayed from CUDA graphs, timed with CUDA events on the
    # launching stream, max over ranks.
    region_ms, launches, per_graph = graph_timed(gpu, step, n_sets,
                                                 args.steps, args.graph_calls)
    # Back-to-back kernels keep the GPU busy, so the kernel's average launch
    # duration is the region over K (an upper bound: it includes the small
    # gaps between kernels).
    kernel_ms = region_ms / args.steps
    clocks = sampler.stop()
    slowest_ms = gpu.max_over_ranks(region_ms)
    ms_per_step = slowest_ms / args.steps
    gpus_active = gpu.busy_gpus(clocks)

    # End to end through the public API: every step copies its inputs in
    # from pinned host memory, runs the operator and copies its result out.
    # Steps are pipelined as a serving loop would run them: the inputs of
    # step i + 1 stream in (copy stream) while step i computes and copies
    # its result out (compute stream, alternating host output buffers).
    host = {name: (None if t is None else t.cpu().contiguous().pin_memory())
            for name, t in zip(('q', 'k', 'v', 'scale', 'key_bias'),
                               w0.tensors())}
    out_hosts = [torch.empty((*w0.q.shape[:3], w0.v.shape[3]),
                             dtype=w0.v.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host.values()
              if t is not None)
    d2h = out_hosts[0].numel() * out_hosts[0].element_size()
    copy_stream = torch.cuda.Stream(dev)
    compute_stream = torch.cuda.Stream(dev)
    # Two device input slots, reused: a slot is refilled only after the
    # step that last read it has finished (no allocation in the loop).
    slots = [{n: (None if t is None else torch.empty(t.shape, dtype=t.dtype,
                                                      device=dev))
              for n, t in host.items()} for _ in range(2)]
    slot_free = [None, None]

    def e2e_step(i):
        d = slots[i % 2]
        with torch.cuda.stream(copy_stream):
            if slot_free[i % 2] is not None:
                copy_stream.wait_event(slot_free[i % 2])
            for n, t in host.items():
                if t is not None:
                    d[n].copy_(t, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(copy_stream)
        compute_stream.wait_event(ready)
        with torch.cuda.stream(compute_stream):
            out = op(d['q'], d['k'], d['v'], d['scale'], d['key_bias'])
            out_hosts[i % 2].copy_(out, non_blocking=True)
            done = torch.cuda.Event()
            done.record(compute_stream)
            slot_free[i % 2] = done

    e2e_steps = max(3, min(args.e2e_steps, args.steps))
    for i in range(2):
        e2e_step(i)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    gpu.barrier()
    e0.record(copy_stream)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(compute_stream)
    torch.cuda.synchronize()
    gpu.barrier()
    e2e_ms = gpu.max_over_ranks(e0.elapsed_time(e1)) / e2e_steps

    # Extras, outside the timed regions: the weak-scaling figure (N > 1,
    # every rank its own full batch) and benchmark config 4 (N == 1).
    extra = {}
    if not args.no_extra and world > 1:
        other = 'weak' if args.scaling == 'strong' else 'strong'
        alt = plan(args.config, other, world)
        del sets
        sets = [make_set(i, other) for i in range(alt['n_sets'])]
        n_sets = alt['n_sets']
        for i in range(3):
            step(i)
        steps_alt = min(args.steps, 500)
        alt_ms, _, _ = graph_timed(gpu, step, n_sets, steps_alt)
        alt_step = gpu.max_over_ranks(alt_ms) / steps_alt
        extra[other] = {'value': alt['global_batch'] / (alt_step * 1e-3),
                        'unit': metric_for(args.config)[1],
                        'ms_per_step': alt_step, 'steps': steps_alt,
                        'queries_per_gpu': alt['per_gpu'],
                        'global_batch': alt['global_batch']}
    if not args.no_extra and world == 1:
        ref_kernel = reference_triton_extra(gpu, sets[:max(1, min(3, len(
            sets)))])
        if ref_kernel is not None:
            if 'ms_per_call' in ref_kernel:
                ref_kernel['this_library_ms_per_call'] = region_ms / args.steps
                ref_kernel['speedup'] = (ref_kernel['ms_per_call'] /
                                         (region_ms / args.steps))
            extra['reference_triton_kernel'] = ref_kernel
    if not args.no_extra and world == 1 and args.config == 2:
        extra['long_sequence'] = long_sequence_extra(gpu)

    # Rank 0 reports.
    metric, unit = metric_for(args.config)
    hbm, tflops_peak, peak_kind = peaks()
    global_batch = p['global_batch']
    if args.config == 4:
        job_flops = flops * global_batch / w0.batch
        value = job_flops / (ms_per_step * 1e-3) / 1e12
        e2e_value = job_flops / (e2e_ms * 1e-3) / 1e12
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        roof = {'bound': 'tensor', 'achieved': achieved,
                'peak': tflops_peak, 'unit': 'TFLOP/s',
                'frac': achieved / tflops_peak, 'traffic': ncu_traffic(4),
                'peak_kind': f'bf16 dense, {peak_kind} (burst)'}
    else:
        value = global_batch / (ms_per_step * 1e-3)
        e2e_value = global_batch / (e2e_ms * 1e-3)
        achieved = alg_bytes / (kernel_ms * 1e-3) / 1e9
        roof = {'bound': 'hbm', 'achieved': achieved, 'peak': hbm,
                'unit': 'GB/s', 'frac': achieved / hbm,
                'traffic': (ncu_traffic(args.config, kernel=args.kernel) *
                            w0.batch / workloads.SHAPES[args.config][0]
                            if ncu_traffic(args.config, kernel=args.kernel)
                            else None),
                'peak_kind': f'HBM copy, {peak_kind}',
                'algorithmic_bytes_per_launch': alg_bytes,
                'vs_8tbs': achieved / 8000.0}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, u, cores, sample = time_cpu(args.config, args.cpu_seconds,
                                       os.cpu_count() or 1)
        cpu = {'value': v, 'unit': u, 'cores': cores, 'kind': 'port',
               'sample': sample, 'cpu_model': cpu_model()}
        if args.config != 4:
            ev, _, _, esample = time_cpu(args.config, args.cpu_seconds / 2,
                                         os.cpu_count() or 1, 'eager')
            cpu['eager'] = {'value': ev, 'unit': u, 'sample': esample}
    if rank == 0:
        line = {
            'metric': metric, 'value': value, 'unit': unit,
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': args.scaling, 'vs_baseline': None,
            'dtype': w0.dtype,
            'data': 'synthetic (seeded; benchmark config shapes and '
                    'distributions)',
            'config': dict(line_config(args, world), **(
                {'shard_of': shards, 'queries_this_gpu': w0.batch}
                if shards != world else {})),
            'launch': {'kernel': vectra_b200.kernel_for(
                           *w0.tensors(), kernel=args.kernel),
                       'graph_calls': per_graph,
                       'queries_this_rank': w0.batch},
            'e2e': {'value': e2e_value, 'unit': unit,
                    'h2d_bytes_per_step': h2d * world,
                    'd2h_bytes_per_step': d2h * world,
                    'h2d_bytes_per_step_per_gpu': h2d,
                    'steps': e2e_steps, 'pipelined': True,
                    # what bounds it: the host->device copy of the inputs
                    'h2d_gbs_per_gpu': h2d / (e2e_ms * 1e-3) / 1e9},
            'gpu_launches': launches,
            'gpu_busy': {'gpus_active': gpus_active, 'n_gpus': world,
                         'basis': 'ranks whose GPU nvidia-smi showed above '
                                  '0% utilisation during the soak and '
                                  'timed region'},
            'kernel_ms_per_launch': kernel_ms,
            'roofline': roof,
            'cpu_baseline': cpu,
            'extra': extra,
            'clocks': clocks,
        }
        emit(line)
    gpu.close()
    return 0


# ---------------------------------------------------------------------------
# Config 5 at the model level (--model)
# ---------------------------------------------------------------------------

MODEL_E2E_CHUNKS = 8    # served batches per end-to-end request
MODEL_SETS = 4          # rotating resident input batches


def load_reference_model_only():
    """The reference's price model (models.price_transformer.model) from its
    unmodified install in baseline/_ref, without the compile pass and
    without this library: the eager model the reference arm times."""
    ref = os.path.join(ROOT, 'baseline', '_ref')
    if not os.path.isfile(os.path.join(ref, 'INSTALL.json')):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from models.price_transformer import model  # pylint: disable=import-outside-toplevel
    return model


def model_batch(args, world):
    w = workloads_module()
    if args.scaling == 'strong':
        return -(-w.PRICE_BATCH // world), w.PRICE_BATCH
    return w.PRICE_BATCH, w.PRICE_BATCH * world


def model_config_line(args, world):
    """The model line's `config`, the same in both arms."""
    w = workloads_module()
    per_gpu, global_batch = model_batch(args, world)
    return {
        'workload': 'config 5 model: the reference PriceTransformer '
                    '(embedding 128, 48 attributes, d_model 256, 4 layers, '
                    '8 heads of 32, ffn 1024, 64 comparables), random init, '
                    f'radius {w.PRICE_RADIUS_KM:g} km',
        'queries_per_gpu': per_gpu, 'global_batch': global_batch,
        'parallelism': f'batch-sharded x{world} ({args.scaling} scaling), '
                       'no collective',
        'l2': 'activations of a batch exceed L2 (17 MB per 65 x 256 bf16 '
              'tensor per 1,024 targets; ~40 live per forward)',
    }


def time_cpu_model(model_lib, seconds, threads, batch=64):
    """The reference's eager price model on the host CPU (float32, the eager
    RBF chain at every site, `threads` intra-op threads) over a fixed
    sample of `batch` targets: (predictions/s, cores, sample)."""
    import torch  # pylint: disable=import-outside-toplevel
    w = workloads_module()
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = model_lib.PriceTransformer(
        model_lib.ModelConfig(**w.PRICE_MODEL)).eval()
    args = w.price_model_inputs(batch, seed=1)
    with torch.no_grad():
        model(*args)  # warm-up
        t0 = time.perf_counter()
        n = 0
        while n == 0 or time.perf_counter() - t0 < seconds:
            model(*args)
            n += 1
        value = n * batch / (time.perf_counter() - t0)
    return value, threads, (f'eager float32 reference model forward, '
                            f'{batch} targets x 65 tokens per pass, '
                            f'{threads} threads')


def run_model_reference(args):
    """The reference arm at the model level: the reference's eager price
    model on the host's cores (its CPU path for config 5: every site runs
    the eager RBF chain)."""
    if int(os.environ.get('RANK', '0')) != 0:
        return 0
    world = int(os.environ.get('WORLD_SIZE', '1'))
    model_lib = load_reference_model_only()
    if model_lib is None:
        emit({'impl': 'reference',
              'unavailable': 'the reference price model is not installed in '
                             'baseline/_ref (no reference checkout at build '
                             'time)'})
        return 0
    metric, unit = metric_for(5, model=True)
    threads = os.cpu_count() or 1
    per_step = max(0.05, min(5.0, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        time_cpu_model(model_lib, per_step / 4, threads)
    runs = [time_cpu_model(model_lib, per_step, threads)
            for _ in range(args.steps)]
    value = float(statistics.median(r[0] for r in runs))
    _, cores, sample = runs[0]
    emit({
        'impl': 'reference', 'metric': metric, 'value': value, 'unit': unit,
        'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': True, 'scaling': args.scaling,
        'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded inputs, random-init weights)',
        'config': model_config_line(args, world),
        'cpu_baseline': {'value': value, 'unit': unit, 'cores': cores,
                         'kind': 'reference', 'sample': sample,
                         'cpu_model': cpu_model(), 'device': 'host CPU'},
        'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    })
    return 0


def run_model(args):
    """Config 5 served whole: the reference's PriceTransformer (4 layers,
    bf16 blocks), compiled by the reference's compile_entry with every RBF
    site rewritten to this library's operator (the one-file swap) and this
    library's value-views pass (vectra_b200.fusion), after the reference's
    numerics gate.

    value: predictions/s with the batches resident in HBM, one step = one
    compiled forward of a served batch (1,024 targets, or the rank's shard
    of them). The forward cannot be captured in a CUDA graph: its radius
    trim is a torch.cond whose predicate Inductor reads on the host. e2e:
    one step = one request of 8 batches from pinned host memory through
    vectra_b200.serving (static slots, pinned staging, copy/compute
    overlap), result read back to the host.
    """
    sys.path.insert(0, ROOT)
    gpu = Gpu(timeout_s=900)
    torch = gpu.torch
    import vectra_b200  # pylint: disable=import-outside-toplevel
    from tests import reference_swap  # pylint: disable=import-outside-toplevel
    from vectra_b200 import serving  # pylint: disable=import-outside-toplevel
    from vectra_b200 import workloads  # pylint: disable=import-outside-toplevel
    world, rank, dev = gpu.world, gpu.rank, gpu.dev

    from vectra_b200 import fusion  # pylint: disable=import-outside-toplevel
    ref = reference_swap.load_reference()
    per_gpu, global_batch = model_batch(args, world)
    cfg = ref.model.ModelConfig(**workloads.PRICE_MODEL)
    spec = ref.compile_entry.ServingSpec(device=str(dev), batch_size=per_gpu,
                                         block_dtype='bfloat16')
    torch.manual_seed(0)
    eager = ref.compile_entry.prepare(ref.model.PriceTransformer(cfg), spec)
    # Served with this library's value-views pass (vectra_b200.fusion:
    # the operator reads V from the projection instead of the copy the
    # reference pass cut at; bit-identical); the reference pass alone is
    # timed too, as extra.reference_pass_only.
    torch._dynamo.reset()  # pylint: disable=protected-access
    plain, plain_report, _ = ref.compile_entry.compile_model(eager, spec)
    torch._dynamo.reset()  # pylint: disable=protected-access
    with fusion.installed() as value_pass:
        compiled, report, compile_s = ref.compile_entry.compile_model(
            eager, spec)
    for r in (plain_report, report):
        if r.sites != cfg.num_layers or r.graph_break_count:
            raise SystemExit(f'compile pass rewrote {r.sites} of '
                             f'{cfg.num_layers} sites with '
                             f'{r.graph_break_count} graph breaks')
    # The reference's serving check before traffic (load_bundle): compiled
    # vs eager on a seeded batch at rtol 1e-3 / atol 1e-3.
    gate, _ = ref.compile_entry.max_abs_error(compiled, eager, cfg, spec,
                                              batches=1)

    def shard(seed):
        full = workloads.price_model_inputs(global_batch if args.scaling ==
                                            'strong' else per_gpu, seed=seed)
        if args.scaling == 'strong':
            lo = min(rank * per_gpu, global_batch - per_gpu)
            full = tuple(t[lo:lo + per_gpu] for t in full)
        return full

    sets = [tuple(t.to(dev) for t in shard(1000 * (args.scaling == 'weak')
                                           * rank + i))
            for i in range(MODEL_SETS)]
    distance = ref.model.microhood.haversine_km(sets[0][2], sets[0][10])
    cheap_branch = bool((sets[0][12] & (distance <= sets[0][5][:, None]))
                        .any(-1).all())
    stream = torch.cuda.current_stream(dev)

    def forward(i):
        with torch.no_grad():
            return compiled(*sets[i % MODEL_SETS])

    for i in range(max(3, args.warmup)):
        forward(i)
    sampler = ClockSampler(gpu.local)
    torch.cuda.synchronize()
    t_soak = time.perf_counter()
    i = 0
    while time.perf_counter() - t_soak < 0.6:
        forward(i)
        i += 1

    # Timed region: exactly K compiled forwards.
    r0 = torch.cuda.Event(enable_timing=True)
    r1 = torch.cuda.Event(enable_timing=True)
    gpu.barrier()
    before = vectra_b200.launch_count()
    r0.record(stream)
    for i in range(args.steps):
        forward(i)
    r1.record(stream)
    torch.cuda.synchronize()
    launches = vectra_b200.launch_count() - before
    gpu.barrier()
    clocks = sampler.stop()
    region_ms = r0.elapsed_time(r1)
    ms_per_step = gpu.max_over_ranks(region_ms) / args.steps
    value = global_batch / (ms_per_step * 1e-3)

    # The reference pass alone (the operator reads the copy of V), the same
    # way, for comparison.
    for i in range(3):
        with torch.no_grad():
            plain(*sets[i % MODEL_SETS])
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    gpu.barrier()
    p0.record(stream)
    for i in range(args.steps):
        with torch.no_grad():
            plain(*sets[i % MODEL_SETS])
    p1.record(stream)
    torch.cuda.synchronize()
    gpu.barrier()
    plain_ms = gpu.max_over_ranks(p0.elapsed_time(p1)) / args.steps
    del plain

    # End to end: requests of 8 served batches from pinned host memory,
    # result read back to the host.
    served = serving.GraphServingModel(compiled, sets[0], capture=False)
    n_e2e = MODEL_E2E_CHUNKS * per_gpu
    host = [t.pin_memory() for t in workloads.price_model_inputs(
        n_e2e, seed=7 + rank)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    e2e_steps = max(3, min(args.e2e_steps, args.steps))
    for _ in range(2):
        served.predict(host).cpu()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    gpu.barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        result = served.predict(host).cpu()
    e1.record(stream)
    torch.cuda.synchronize()
    gpu.barrier()
    d2h = result.numel() * result.element_size()
    e2e_ms = gpu.max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    e2e_value = MODEL_E2E_CHUNKS * global_batch / (e2e_ms * 1e-3)

    # The site kernel on its own, on the sites' shapes (benchmark config 5's
    # site workload at the rank's batch), event-timed over back-to-back
    # calls.
    hbm, _, peak_kind = peaks()
    site_sets = [workloads.make(5, device=dev, seed=i, batch=per_gpu)
                 for i in range(4)]
    op = torch.ops.vectra.rbf_attention
    for w in site_sets:
        op(*w.tensors())
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    n_site = 200
    s0.record(stream)
    for i in range(n_site):
        op(*site_sets[i % 4].tensors())
    s1.record(stream)
    torch.cuda.synchronize()
    site_ms = s0.elapsed_time(s1) / n_site
    alg_bytes = workloads.algorithmic_bytes(site_sets[0])
    achieved = alg_bytes / (site_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = time_cpu_model(ref.model, args.cpu_seconds,
                                          os.cpu_count() or 1)
        cpu = {'value': v, 'unit': 'predictions/s', 'cores': cores,
               'kind': 'reference', 'sample': sample,
               'cpu_model': cpu_model()}
    if rank == 0:
        metric, unit = metric_for(5, model=True)
        emit({
            'metric': metric, 'value': value, 'unit': unit, 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': args.scaling, 'vs_baseline': None, 'dtype': 'bf16',
            'data': 'synthetic (seeded inputs, random-init weights)',
            'config': model_config_line(args, world),
            'extra': {'reference_pass_only': {
                'ms_per_step': plain_ms,
                'value': global_batch / (plain_ms * 1e-3),
                'note': 'the reference compile pass alone: the operator '
                        'reads the contiguous copy of V'}},
            'compile': {'sites': report.sites, 'matches': report.matches,
                        'value_views_rewired': value_pass.rewired,
                        'graph_count': report.graph_count,
                        'graph_break_count': report.graph_break_count,
                        'seconds': compile_s,
                        'numerics_gate_max_abs_error': gate,
                        'radius_branch': ('within_radius (cheap)'
                                          if cheap_branch else
                                          'with_fallback')},
            'e2e': {'value': e2e_value, 'unit': unit,
                    'h2d_bytes_per_step': h2d * world,
                    'd2h_bytes_per_step': d2h * world,
                    'steps': e2e_steps,
                    'targets_per_step': MODEL_E2E_CHUNKS * global_batch,
                    'serving': 'vectra_b200.serving.GraphServingModel, '
                               '2 slots, capture=False'},
            'gpu_launches': launches,
            'roofline': {
                'bound': 'hbm', 'achieved': achieved, 'peak': hbm,
                'unit': 'GB/s', 'frac': achieved / hbm,
                'traffic': ncu_traffic(5),
                'peak_kind': f'HBM copy, {peak_kind}',
                'kernel': 'rbf_small, one site, timed alone',
                'algorithmic_bytes_per_launch': alg_bytes,
                'site_ms': site_ms,
                'sites_share_of_forward': cfg.num_layers * site_ms /
                                          ms_per_step},
            'cpu_baseline': cpu,
            'clocks': clocks,
        })
    del served
    gpu.close()
    return 0


# ---------------------------------------------------------------------------
# The index-shard scan path (--scan l2|pq)
# ---------------------------------------------------------------------------

# Queries per step: a CTA's group of 8 for L2 (the distances stay under the
# HBM time), one for PQ (its table lookups grow with the queries and would
# outrun the 256 MB of codes).
SCAN_QUERIES = {'l2': 8, 'pq': 1}
SCAN_K = 64          # the reference's rerank_depth default
SCAN_L2 = dict(rows=1 << 20, dim=128)          # 512 MB of float32 rows
SCAN_PQ = dict(rows=1 << 24, subspaces=16)     # 256 MB of codes


def scan_metric(kind):
    if kind == 'l2':
        return (f'exhaustive L2 top-{SCAN_K} scan queries/s (shard of '
                f'{SCAN_L2["rows"]:,} rows x {SCAN_L2["dim"]} float32, '
                f'{SCAN_QUERIES["l2"]} queries per step)', 'queries/s')
    return (f'PQ-ADC top-{SCAN_K} scan queries/s (shard of '
            f'{SCAN_PQ["rows"]:,} codes x {SCAN_PQ["subspaces"]} bytes, '
            f'{SCAN_QUERIES["pq"]} query per step)', 'queries/s')


def scan_inputs(kind, seed=0):
    """Seeded host arrays of the scan workload (rows or codes, queries or
    tables)."""
    rng = np.random.default_rng(seed)
    if kind == 'l2':
        rows = rng.standard_normal((SCAN_L2['rows'], SCAN_L2['dim']),
                                   dtype=np.float32)
        queries = rng.standard_normal((4 * SCAN_QUERIES['l2'],
                                       SCAN_L2['dim']), dtype=np.float32)
        return rows, queries
    codes = rng.integers(0, 256, (SCAN_PQ['rows'], SCAN_PQ['subspaces']),
                         dtype=np.uint8)
    tables = (rng.random((4 * SCAN_QUERIES['pq'], SCAN_PQ['subspaces'], 256),
                         dtype=np.float32) * 4)
    return codes, tables


def time_scan_cpu(kind, data, queries, seconds, threads):
    """The reference's scan on the host: ExhaustiveSearch's bounded top-k
    over L2SquaredDistance / PqAdcDistance from oracle/_ref (the reference
    engine's own sources) when built, else the NumPy port; one query per
    thread over a bounded sample of the shard. (queries/s, cores, kind,
    sample)."""
    from oracle import scan_oracle  # pylint: disable=import-outside-toplevel
    ref = scan_oracle.load_reference(fast=True) or scan_oracle.load_reference()
    n_sample = min(data.shape[0], 1 << 18)
    sample = np.ascontiguousarray(data[:n_sample])
    if ref is not None:
        one = ((lambda q: ref.exhaustive_topk(q, sample, SCAN_K))
               if kind == 'l2' else
               (lambda q: ref.pq_topk(q, sample, SCAN_K)))
        kind_name = 'reference'
    else:
        one = ((lambda q: scan_oracle.exhaustive_l2_topk(q, sample, SCAN_K))
               if kind == 'l2' else
               (lambda q: scan_oracle.pq_topk(q, sample, SCAN_K)))
        kind_name = 'port'
    scale = data.shape[0] / n_sample  # full-shard queries per sampled query
    with concurrent.futures.ThreadPoolExecutor(threads) as pool:
        list(pool.map(one, [queries[i % len(queries)]
                            for i in range(threads)]))  # warm-up
        t0 = time.perf_counter()
        done = 0
        while done == 0 or time.perf_counter() - t0 < seconds:
            list(pool.map(one, [queries[(done + i) % len(queries)]
                                for i in range(threads)]))
            done += threads
        elapsed = time.perf_counter() - t0
    sample_txt = (f'{kind_name}: one query per thread over the first '
                  f'{n_sample:,} rows of the shard ({done} queries), scaled '
                  f'to the full shard')
    return done / scale / elapsed, threads, kind_name, sample_txt


def scan_launches(n_cand, k):
    """Kernel launches of one scan call: a level kernel and a select per
    level, plus the warp-list re-scan's two (which return at once unless a
    query's last level overflowed). Mirrors the level plan in
    vectra_b200/csrc/scan.cu (plan_for)."""
    cap, sample0 = 32768, 8192
    if n_cand <= cap:
        return 2
    levels, s = 1, sample0
    while levels < 6 and k * n_cand > (cap // 4) * s:
        enough = -(-k * n_cand // (cap // 4))
        s2 = -(-min(enough, s * (cap // 8) // k) // 32) * 32
        if 2 * s2 >= n_cand:
            break
        levels += 1
        s = s2
    return 2 * (levels + 1) + 2


def run_scan_reference(args):
    if int(os.environ.get('RANK', '0')) != 0:
        return 0
    sys.path.insert(0, ROOT)
    metric, unit = scan_metric(args.scan)
    data, queries = scan_inputs(args.scan)
    threads = os.cpu_count() or 1
    per_step = max(0.2, min(10.0, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        time_scan_cpu(args.scan, data, queries, per_step / 4, threads)
    runs = [time_scan_cpu(args.scan, data, queries, per_step, threads)
            for _ in range(args.steps)]
    value = float(statistics.median(r[0] for r in runs))
    _, cores, kind, sample = runs[0]
    emit({
        'impl': 'reference', 'metric': metric, 'value': value, 'unit': unit,
        'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
        'dtype': 'f32', 'data': 'synthetic (seeded)',
        'config': {'workload': f'scan {args.scan}', 'device': 'host CPU',
                   'threads': cores},
        'cpu_baseline': {'value': value, 'unit': unit, 'cores': cores,
                         'kind': kind, 'sample': sample,
                         'cpu_model': cpu_model()},
        'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    })
    return 0


def run_scan(args):
    """The shard (rows or PQ codes) resident in HBM; one step = one call of
    the scan over SCAN_QUERIES queries, through the C ABI with the argument
    block prepared once (queries rotate over four sets). The shard (> L2)
    is read from HBM by every step. e2e: the same with the step's queries
    copied in from pinned host memory and its results read back."""
    import ctypes  # pylint: disable=import-outside-toplevel
    import torch  # pylint: disable=import-outside-toplevel
    import torch.distributed as dist  # pylint: disable=import-outside-toplevel
    sys.path.insert(0, ROOT)
    from vectra_b200 import _lib  # pylint: disable=import-outside-toplevel
    from vectra_b200 import scan  # pylint: disable=import-outside-toplevel
    from vectra_b200 import sharding  # pylint: disable=import-outside-toplevel

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    distributed = world > 1
    if distributed:
        import datetime  # pylint: disable=import-outside-toplevel
        dist.init_process_group('nccl', device_id=dev,
                                timeout=datetime.timedelta(seconds=300))

    def barrier():
        if distributed:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    data_h, queries_h = scan_inputs(args.scan, seed=rank)
    data = torch.from_numpy(data_h).to(dev)
    queries = torch.from_numpy(queries_h).to(dev)
    nq, k = SCAN_QUERIES[args.scan], SCAN_K
    ws = torch.empty(scan.workspace_bytes(nq, data.shape[0], k),
                     dtype=torch.uint8, device=dev)
    out_d = torch.empty(nq, k, dtype=torch.float32, device=dev)
    out_n = torch.empty(nq, k, dtype=torch.int32, device=dev)
    counts = torch.empty(nq, dtype=torch.int32, device=dev)
    res = scan.Results(out_d.data_ptr(), out_n.data_ptr(), counts.data_ptr())
    cand = scan.Candidates(None, None, 0)
    if args.scan == 'l2':
        alg_bytes = data.numel() * 4 + nq * data.shape[1] * 4 + nq * k * 8
        blocks = [scan.L2Args(queries[i * nq].data_ptr(), nq,
                              queries.stride(0), data.data_ptr(),
                              data.shape[0], data.stride(0), data.shape[1],
                              k, cand, res, ws.data_ptr(), ws.numel())
                  for i in range(4)]
        call = _lib.LIB.vectra_scan_l2_topk
    else:
        alg_bytes = data.numel() + nq * queries[0].numel() * 4 + nq * k * 8
        blocks = [scan.PqArgs(queries[i * nq].data_ptr(), nq, data.data_ptr(),
                              data.shape[0], data.stride(0), data.shape[1], k,
                              cand, res, ws.data_ptr(), ws.numel())
                  for i in range(4)]
        call = _lib.LIB.vectra_scan_pq_topk
    stream = torch.cuda.current_stream(dev)
    handle = ctypes.c_void_p(stream.cuda_stream)
    # A level kernel and a select per level, then the re-scan check.
    launches_per_step = scan_launches(data.shape[0], SCAN_K)

    def step(i):
        status = call(ctypes.byref(blocks[i % 4]), handle)
        if status != _lib.OK:
            raise RuntimeError(_lib.strerror(status))

    for i in range(max(3, args.warmup)):
        step(i)
    if args.profile:
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        if distributed:
            dist.destroy_process_group()
        return 0
    sampler = ClockSampler(local)
    t_soak = time.perf_counter()
    i = 0
    while time.perf_counter() - t_soak < 0.6:
        step(i)
        i += 1
        if i % 16 == 0:
            torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    region_ms = e0.elapsed_time(e1)
    ms_per_step = sharding.max_over_ranks(region_ms, device=dev) / args.steps
    value = nq * world / (ms_per_step * 1e-3)

    # End to end: each step's queries (or tables) from pinned host memory
    # into the argument block's buffer, the results back to pinned host
    # memory.
    q_host = torch.from_numpy(queries_h[:nq]).pin_memory()
    d_host = torch.empty_like(out_d, device='cpu').pin_memory()
    n_host = torch.empty_like(out_n, device='cpu').pin_memory()
    h2d = q_host.numel() * q_host.element_size()
    d2h = (d_host.numel() * d_host.element_size() +
           n_host.numel() * n_host.element_size())
    target = queries[:nq]
    e2e_steps = max(3, min(args.e2e_steps, args.steps))
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    barrier()
    f0.record(stream)
    for _ in range(e2e_steps):
        target.copy_(q_host, non_blocking=True)
        step(0)
        d_host.copy_(out_d, non_blocking=True)
        n_host.copy_(out_n, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = sharding.max_over_ranks(f0.elapsed_time(f1),
                                     device=dev) / e2e_steps
    hbm, _, peak_kind = peaks()
    achieved = alg_bytes / (ms_per_step * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, kind, sample = time_scan_cpu(args.scan, data_h, queries_h,
                                               args.cpu_seconds,
                                               os.cpu_count() or 1)
        cpu = {'value': v, 'unit': 'queries/s', 'cores': cores, 'kind': kind,
               'sample': sample, 'cpu_model': cpu_model()}
    if rank == 0:
        metric, unit = scan_metric(args.scan)
        emit({
            'metric': metric, 'value': value, 'unit': unit, 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded)',
            'config': {
                'workload': f'scan {args.scan}: one shard per GPU, '
                            f'{nq} queries per step, k = {k}',
                'shard_bytes': data.numel() * data.element_size(),
                'l2': 'shard > L2, read from HBM every step',
                'parallelism': f'a shard per GPU x{world}, no collective',
            },
            'e2e': {'value': nq * world / (e2e_ms * 1e-3), 'unit': unit,
                    'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
                    'steps': e2e_steps},
            'gpu_launches': launches_per_step * args.steps,
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm,
                         'unit': 'GB/s', 'frac': achieved / hbm,
                         'traffic': ncu_traffic(
                             None, 'scan_levels',
                             f'dram_bytes_full_level_{args.scan}'),
                         'peak_kind': f'HBM copy, {peak_kind}',
                         'algorithmic_bytes_per_launch': alg_bytes,
                         'kernel': 'every launch of a step (sample and '
                                   'full levels, selects, re-scan check)'},
            'cpu_baseline': cpu,
            'clocks': clocks,
        })
    if distributed:
        dist.destroy_process_group()
    return 0


# The JSON line goes to the process's original standard output; while the
# benchmark runs, file descriptor 1 points at standard error, so that what
# libraries print there (NCCL's version banner, for one) cannot come before
# or between the lines a driver parses.
_RESULT_OUT = None


def emit(line):
    out = _RESULT_OUT or sys.stdout
    out.write(json.dumps(line) + '\n')
    out.flush()


def main(argv=None):
    global _RESULT_OUT  # pylint: disable=global-statement
    args = parse_args(argv)
    sys.stdout.flush()
    saved = os.dup(1)
    try:
        _RESULT_OUT = os.fdopen(os.dup(saved), 'w')
        os.dup2(2, 1)
        if args.impl == 'reference':
            if args.scan:
                return run_scan_reference(args)
            return (run_model_reference(args) if args.model
                    else run_reference(args))
        if args.scan:
            return run_scan(args)
        return run_model(args) if args.model else run_vectra(args)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
        if _RESULT_OUT is not None:
            _RESULT_OUT.close()
            _RESULT_OUT = None


if __name__ == '__main__':
    sys.exit(main())
