"""Contextualizer forward benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|triton]
                    [--config c2|c3|c4|c5]

A step is one contextualizer forward over one batch of synthetic input shaped
like a BASELINE config (default c2: Avey causal, bf16, B=64 per GPU, N=512,
head/tail d'=768, bias and gate). With N GPUs (one process per GPU under
torchrun) every rank runs its own batch shard: no collective on the data path
("scaling": "weak" for c2-c4; c5 keeps the global batch of 1024 fixed and
splits it, "strong").

value  device time: K steps replayed from CUDA graphs between CUDA events on
       the launching stream, inputs resident in HBM and rotating over three
       sets larger than L2; whole-job tokens/s over the max across ranks.
e2e    the same metric through the public API (avey / avey_b) with pinned
       host buffers: every step copies its inputs host->device and reads the
       output back, inside the timed region.
--impl reference  times the reference's own CPU implementation of the path:
       avey_kernels.ops.avey / avey_b with backend='torch' (its _reference,
       fp32) from the unmodified install in baseline/_ref, on CPU tensors of
       the whole per-GPU batch, every host thread, up to K steps within about
       a minute; rank 0 only, the line stating the same global workload as
       the GPU arm. Without baseline/_ref: the NumPy port in oracle/.
cpu_baseline  (in the GPU arm's line, one GPU) the NumPy port of _reference
       (oracle/, fp32, all host threads) on one batch row per run, ~10 s.
--impl triton  (informational, one GPU) times the reference's own GPU kernel
       through its public API (avey_kernels.ops, backend='triton', from the
       unmodified install in baseline/_ref): normalisation pre-pass,
       contiguous copies and the Triton mix kernel, device time with CUDA
       events over K calls on the same inputs as --impl ours.
--pass train  (informational, one GPU) a step is one forward plus backward
       (gradients of x, W and bias for an upstream gradient of the output's
       shape): --impl ours runs the native forward and backward, --impl
       reference the reference's only differentiable path (autograd through
       avey_kernels.ops._reference, backend='torch', from baseline/_ref) on
       the same GPU and inputs. Metric 'contextualizer fwd+bwd tokens/s'.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (batch per GPU or global, context, features, op, causal, bias, ragged, boost, scaling;
    # dtype bf16 unless given)
    'c1': dict(batch=2, n=256, d=128, op='avey', bias=True, zero_bias=True, ragged=False,
               boost=False, scaling='weak', dtype='f32',
               desc="Avey causal, fp32, B=2 per GPU, N=256, d'=128, bias 0 (8-row CUDA-core "
                    "kernel on CTA pairs)"),
    'c2f32': dict(batch=64, n=512, d=768, op='avey', bias=True, ragged=False, boost=False,
                  scaling='weak', dtype='f32',
                  desc="config 2's shape in fp32 (3xTF32 tensor cores): Avey causal, B=64 per GPU, "
                       "N=512, d'=768"),
    'c2': dict(batch=64, n=512, d=768, op='avey', bias=True, ragged=False, boost=False,
               scaling='weak', desc='Avey causal contextualizer, bf16, B=64 per GPU, N=512, '
                                    "head/tail d'=768, W_mix~N(0,0.02), bias~N(0,0.01)"),
    'c3': dict(batch=128, n=512, d=384, op='avey_b', bias=False, ragged=True, boost=False,
               scaling='weak', desc='Avey-B bidirectional, bf16, B=128 per GPU, N=512, '
                                    "d'=384, padding lengths ~U[N/4, N]"),
    'c4': dict(batch=16, n=2048, d=1024, op='avey', bias=False, ragged=False, boost=True,
               scaling='weak', desc="Long-context Avey causal, bf16, B=16 per GPU, N=2048, d'=1024,"
                                    ' 5% rows x50'),
    'c5': dict(batch=1024, n=512, d=768, op='avey', bias=False, ragged=False, boost=False,
               scaling='strong', desc='Avey causal bf16, global B=1024 split by batch, N=512, '
                                      "d'=768"),
}
METRIC = 'contextualizer fwd tokens/s'
UNIT = 'tokens/s'


def load_peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        p = json.loads(path.read_text())
        return dict(hbm_gbs=p['hbm_gbs'], bf16_tflops=p['bf16_tflops'],
                    bf16_tflops_sustained=p.get('bf16_tflops_sustained'), source='measured')
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0,
                source='fallback')


def rank_env():
    from avey_kernel_b200.shard import rank_env as env
    return env()


def shard_batch(cfg, world):
    """Batch rows per rank: fixed per GPU (weak scaling) or the global batch
    split evenly (strong scaling, config 5)."""
    if cfg['scaling'] == 'strong':
        from avey_kernel_b200.shard import shard_bounds
        try:
            start, stop = shard_bounds(cfg['batch'], world, 0)
        except ValueError as e:
            raise SystemExit(str(e))
        return stop - start
    return cfg['batch']


def make_inputs(cfg, batch, seed, device='cpu'):
    """Seeded synthetic inputs (fixed draw order: x, W, bias, lengths, boost).
    Inputs of more than 2^28 elements (config 5's 1024-row batch on one GPU)
    draw x on the device with a seeded CUDA generator: the same distribution,
    without minutes of host-side generation."""
    import torch
    g = torch.Generator().manual_seed(seed)
    n, d = cfg['n'], cfg['d']
    if device != 'cpu' and batch * n * 2 * d > (1 << 28):
        gd = torch.Generator(device=device).manual_seed(seed)
        x = torch.randn(batch, n, 2 * d, generator=gd, device=device)
    else:
        x = torch.randn(batch, n, 2 * d, generator=g)
    w = torch.randn(n, n, generator=g) * 0.02
    bias = torch.randn(d, generator=g) * 0.01 if cfg['bias'] else None
    if bias is not None and cfg.get('zero_bias'):
        bias = torch.zeros(d)
    valid = None
    if cfg['ragged']:
        lengths = torch.randint(n // 4, n + 1, (batch,), generator=g)
        valid = torch.arange(n)[None, :] < lengths[:, None]
    if cfg['boost']:
        rows = (torch.rand(batch, n, 1, generator=g) < 0.05).to(x.device)
        x = torch.where(rows, x * 50, x)
    bf = torch.float32 if cfg.get('dtype') == 'f32' else torch.bfloat16
    out = dict(x=x.to(bf), w=w.to(bf) if cfg['op'] == 'avey' else None,
               bias=bias.to(bf) if bias is not None else None, valid=valid)
    if device != 'cpu':
        out = {k: (v.to(device) if v is not None else None) for k, v in out.items()}
    return out


def algorithmic(cfg, batch, valid):
    """Bytes and useful FLOPs of one launch: z_tr, z_tl read, out written, V,
    bias, valid; 4 d' FLOPs per allowed (query, key) pair."""
    import numpy as np
    n, d, es = cfg['n'], cfg['d'], 4 if cfg.get('dtype') == 'f32' else 2
    causal = cfg['op'] == 'avey'
    if valid is None:
        pairs = batch * (n * (n + 1) // 2 if causal else n * n)
    else:
        ok = valid.cpu().numpy().astype(bool)
        cnt = ok.sum(axis=1).astype(np.int64)
        pairs = int((cnt * cnt).sum()) if not causal else int(
            (np.cumsum(ok, axis=1) * ok).sum())
    nbytes = es * batch * n * d * 3 + (es * n * n if causal else 0) + (es * d if cfg['bias'] else 0)
    nbytes += batch * n if valid is not None else 0
    return nbytes, 4 * d * pairs


def nvml_handle(nv, cuda_index):
    """NVML handle of a CUDA device (CUDA_VISIBLE_DEVICES may renumber GPUs)."""
    import torch
    props = torch.cuda.get_device_properties(cuda_index)
    uuid = getattr(props, 'uuid', None)
    if uuid is not None:
        text = str(uuid)
        for cand in (text if text.startswith('GPU-') else 'GPU-' + text, text):
            try:
                return nv.nvmlDeviceGetHandleByUUID(cand)
            except Exception:
                pass
    bus = getattr(props, 'pci_bus_id', None)
    if bus is not None:
        pci = (f'{getattr(props, "pci_domain_id", 0):08x}:{bus:02x}:'
               f'{getattr(props, "pci_device_id", 0):02x}.0')
        try:
            return nv.nvmlDeviceGetHandleByPciBusId(pci)
        except Exception:
            pass
    return nv.nvmlDeviceGetHandleByIndex(cuda_index)


class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML."""

    REASONS = {  # NVML clocks-event reason bits
        0x1: 'gpu_idle', 0x2: 'applications_clocks_setting', 0x4: 'sw_power_cap',
        0x8: 'hw_slowdown', 0x10: 'sync_boost', 0x20: 'sw_thermal_slowdown',
        0x40: 'hw_thermal_slowdown', 0x80: 'hw_power_brake_slowdown',
        0x100: 'display_clock_setting',
    }

    def __init__(self, index, period=0.01):
        self.index, self.period = index, period
        self.samples, self.error = [], None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = nvml_handle(pynvml, self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as exc:  # pragma: no cover - reported, not fatal
            self.error = repr(exc)
            self.max_mhz = None
        return self

    def _sample(self):
        nv = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        power = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
        self.samples.append((sm, reasons, power))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception as exc:  # pragma: no cover
                self.error = repr(exc)
                return
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': self.max_mhz, 'reasons': [],
                    'samples': 0, 'error': self.error}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = 0
        for s in busy:
            reasons |= s[1]
        names = [name for bit, name in self.REASONS.items() if reasons & bit and bit != 0x1]
        return {'sm_mhz': statistics.median(s[0] for s in busy), 'sm_max_mhz': self.max_mhz,
                'reasons': names, 'samples': len(self.samples),
                'power_w_max': max(s[2] for s in self.samples)}


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        info = threadpool_info()
        if info:
            return max(i.get('num_threads', 1) for i in info)
    except Exception:
        pass
    return host_cores()


class all_host_threads:
    """Let the BLAS pools use every core this process may run on (torchrun
    exports OMP_NUM_THREADS=1 to its children)."""

    def __enter__(self):
        self._ctl = None
        try:
            from threadpoolctl import threadpool_limits
            self._ctl = threadpool_limits(limits=host_cores())
        except Exception:
            pass
        return self

    def __exit__(self, *exc):
        if self._ctl is not None:
            self._ctl.restore_original_limits()


def time_cpu_port(cfg, seconds=10.0, max_steps=None, warmup=1, rows=1):
    """Time the NumPy port of the reference (oracle/, fp32 accumulation, all
    BLAS threads) on `rows` batch rows per step. Returns tokens/s, steps, rows."""
    import numpy as np
    import oracle
    inp = make_inputs(cfg, rows, seed=0)
    d = cfg['d']
    x = inp['x'].float().numpy()
    zl, zt = x[..., :d], x[..., d:]
    w = inp['w'].float().numpy() if inp['w'] is not None else None
    bias = inp['bias'].float().numpy() if inp['bias'] is not None else None
    valid = inp['valid'].numpy() if inp['valid'] is not None else None

    def step():
        if cfg['op'] == 'avey':
            return oracle.avey(zt, w, z_tl=zl, bias=bias, valid=valid, accum=np.float32)
        return oracle.avey_b(zt, z_tl=zl, bias=bias, valid=valid, accum=np.float32)

    for _ in range(warmup):
        step()
    times = []
    t_end = time.perf_counter() + seconds
    while (max_steps is None and time.perf_counter() < t_end) or (
            max_steps is not None and len(times) < max_steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    tokens = rows * cfg['n']
    return tokens / statistics.median(times), len(times), sum(times)


def time_reference_torch(cfg, batch, steps, warmup, budget_s=60.0):
    """Time the reference's own CPU path: avey_kernels.ops.avey / avey_b with
    backend='torch' (its _reference: inputs upcast to fp32, dense S) from the
    unmodified install in baseline/_ref, on CPU tensors of the whole per-GPU
    batch, with every host core. Returns (tokens/s, steps timed, seconds,
    threads), or None when baseline/_ref does not import."""
    try:
        sys.path.insert(0, str(ROOT / 'baseline' / '_ref'))
        from avey_kernels import ops as ref_ops
    except Exception:
        return None
    import torch
    torch.set_num_threads(host_cores())
    inp = make_inputs(cfg, batch, seed=0)
    d = cfg['d']
    # The reference's callers pass the head and tail halves as separate tensors.
    head, tail = inp['x'][..., :d].contiguous(), inp['x'][..., d:].contiguous()

    def step():
        with torch.no_grad():
            if cfg['op'] == 'avey':
                return ref_ops.avey(tail, inp['w'], z_tl=head, bias=inp['bias'], valid=inp['valid'],
                                    backend='torch')
            return ref_ops.avey_b(tail, z_tl=head, bias=inp['bias'], valid=inp['valid'],
                                  backend='torch')

    for _ in range(max(1, min(warmup, 2))):
        step()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < steps and (len(times) < 3 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return batch * cfg['n'] / statistics.median(times), len(times), sum(times), torch.get_num_threads()


def run_reference(args, cfg):
    world, rank, _ = rank_env()
    if rank != 0:
        return 0  # the CPU reference arm runs once, on rank 0
    batch = shard_batch(cfg, world)
    t0 = time.perf_counter()
    ref = time_reference_torch(cfg, batch, steps=args.steps, warmup=args.warmup)
    if ref is not None:
        value, steps, busy, cores = ref
        kind = 'reference'
        sample = (f'{steps} timed steps of the whole per-GPU batch ({batch} x {cfg["n"]} tokens) of '
                  f'{args.config}, {busy:.1f} s: avey_kernels.ops.{cfg["op"]}(..., backend="torch") '
                  f'from baseline/_ref (the reference\'s _reference, fp32) on CPU tensors')
        dtype = 'f32' if cfg.get('dtype') == 'f32' else 'bf16 inputs, f32 arithmetic'
    else:
        with all_host_threads():
            value, steps, busy = time_cpu_port(cfg, max_steps=args.steps, warmup=args.warmup, rows=1)
            cores = cpu_threads()
        kind = 'port'
        sample = (f'{steps} steps x 1 of {batch} batch rows ({cfg["n"]} tokens) of {args.config}, '
                  f'fp32 NumPy port of avey_kernels/ops.py::_reference (oracle/); baseline/_ref '
                  f'was not importable')
        dtype = 'f32'
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1e3 * batch * cfg['n'] / value,
        'higher_is_better': True, 'scaling': cfg['scaling'], 'vs_baseline': None,
        'dtype': dtype, 'data': 'synthetic',
        # The same workload as the GPU arm's line: at N GPUs the job is N per-GPU
        # batches; the host's cores process it at this rate whatever N is.
        'config': {'workload': f'{args.config}: {cfg["desc"]}', 'context': cfg['n'],
                   'features': cfg['d'], 'batch_per_gpu': batch,
                   'global_batch': batch * world, 'parallelism': f'host CPU, {cores} threads'},
        'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': kind,
                         'sample': sample},
        'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
        'wall_s': time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, cfg):
    import torch
    import torch.distributed as dist
    from avey_kernel_b200 import _native, avey, avey_b, ops

    world, rank, local = rank_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device('cuda', torch.cuda.current_device())
    batch = shard_batch(cfg, world)
    d = cfg['d']
    peaks = load_peaks()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    # Three input sets (each > 1/3 of L2) rotate so no step finds its inputs in L2.
    nsets = 3
    sets = [make_inputs(cfg, batch, seed=1000 * rank + s, device=dev) for s in range(nsets)]
    outs = [None] * nsets

    def call(s):
        t = sets[s]
        head, tail = t['x'][..., :d], t['x'][..., d:]
        if cfg['op'] == 'avey':
            return avey(tail, t['w'], z_tl=head, bias=t['bias'], valid=t['valid'])
        return avey_b(tail, z_tl=head, bias=t['bias'], valid=t['valid'])

    t0 = time.perf_counter()
    # Verification first (outside any timed region): sampled rows vs the oracle.
    import numpy as np
    import oracle
    y = call(0)
    torch.cuda.synchronize()
    t = sets[0]
    verify_err = 0.0
    for r in sorted({0, batch - 1}):
        x = t['x'][r:r + 1].float().cpu().numpy()
        kw = dict(z_tl=x[..., :d], bias=t['bias'].float().cpu().numpy() if t['bias'] is not None else None,
                  valid=t['valid'][r:r + 1].cpu().numpy() if t['valid'] is not None else None)
        ref = (oracle.avey(x[..., d:], t['w'].float().cpu().numpy(), **kw) if cfg['op'] == 'avey'
               else oracle.avey_b(x[..., d:], **kw))
        got = y[r:r + 1].float().cpu().numpy()
        verify_err = max(verify_err, float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30)))
    # Gather each rank's first output row to rank 0 (verification only, NCCL).
    from avey_kernel_b200.shard import gather_to_rank0, max_over_ranks
    gathered = gather_to_rank0(y[0])
    if rank == 0 and gathered is not None:
        assert len(gathered) == world and all(torch.isfinite(g.float()).all() for g in gathered)
    verify_err = max_over_ranks(verify_err, device=dev)
    plan = ops.plan(sets[0]['x'][..., d:], sets[0]['w'], sets[0]['x'][..., :d], sets[0]['bias'],
                    sets[0]['valid'], causal=cfg['op'] == 'avey', normalize=cfg['op'] != 'avey')
    kernel_name = {1: 'simt_contextualize', 2: 'tc_contextualize (whole step)'}[plan.kernel]
    if plan.kernel == 2 and plan.launches == 3:  # contexts above 512: two tensor-core kernels
        # O = P Z on the batched GEMM without a padding mask, on tc_pv with one.
        mix = 'tc_pv' if sets[0]['valid'] is not None else 'tc_gemm (O = P Z)'
        kernel_name = f'norm_prepass + tc_gram_p + {mix} (whole step)'
    f32 = cfg.get('dtype') == 'f32'
    if plan.kernel == 2 and f32:  # fp32: the 3xTF32 pair, no pre-pass
        kernel_name = 'tf_gram_p + tf_pv (whole step)'
    if plan.reason == _native.REASON_SMALL:  # small fp32 problems: the 8-row CUDA-core kernel
        kernel_name = 'small_contextualize (whole step)'

    # Warm-up (untimed), then capture chunks of steps into CUDA graphs.
    for i in range(max(args.warmup, 3)):
        outs[i % nsets] = call(i % nsets)
    torch.cuda.synchronize()
    chunk = min(args.steps, 60)
    graphs = []
    remaining = args.steps
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    launches_captured = 0
    keep = []
    while remaining > 0:
        n_steps = min(chunk, remaining)
        if graphs and n_steps == graphs[0][1]:
            graphs.append((graphs[0][0], n_steps))
        else:
            g = torch.cuda.CUDAGraph()
            before = _native.launch_count()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n_steps):
                    keep.append(call(i % nsets))
            launches_captured += _native.launch_count() - before
            graphs.append((g, n_steps))
        remaining -= n_steps
    torch.cuda.synchronize()
    gpu_launches = sum(n for _, n in graphs) * plan.launches  # native kernels per step
    for g, _ in graphs[:2]:  # warm the graph executables
        g.replay()
    torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for g, _ in graphs:
                g.replay()
            end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_total = start.elapsed_time(end)
    ms_step = max_over_ranks(ms_total / args.steps, device=dev)
    tokens_per_step = batch * cfg['n'] * world
    value = tokens_per_step / (ms_step / 1e3)

    # End to end through the public API with pinned host buffers. Every step
    # copies its inputs host->device, calls avey/avey_b and copies the output
    # back; consecutive steps overlap on three streams (copy-in of step i+1,
    # compute of step i, copy-out of step i-1), with two device input buffers
    # and two pinned output buffers, as a throughput-bound caller would run it.
    e2e_steps = max(3, min(args.steps, 30))
    t = sets[0]
    x_host = t['x'].cpu().pin_memory()
    w_host = t['w'].cpu().pin_memory() if t['w'] is not None else None
    b_host = t['bias'].cpu().pin_memory() if t['bias'] is not None else None
    v_host = t['valid'].cpu().pin_memory() if t['valid'] is not None else None
    hosts = (x_host, w_host, b_host, v_host)
    out_host = [torch.empty(batch, cfg['n'], d, dtype=t['x'].dtype).pin_memory() for _ in range(2)]
    dev_bufs = [[torch.empty(h.shape, dtype=h.dtype, device=dev) if h is not None else None
                 for h in hosts] for _ in range(2)]
    h2d = sum(h.numel() * h.element_size() for h in hosts if h is not None)
    d2h = out_host[0].numel() * out_host[0].element_size()
    s_cmp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        k = i % 2
        xd, wd, bd, vd = dev_bufs[k]
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_cmp[k])  # step i-2 has finished reading buffer k
            for dst, src in zip(dev_bufs[k], hosts):
                if src is not None:
                    dst.copy_(src, non_blocking=True)
            ev_in[k].record(s_in)
        s_cmp.wait_event(ev_in[k])
        head, tail = xd[..., :d], xd[..., d:]
        if cfg['op'] == 'avey':
            o = avey(tail, wd, z_tl=head, bias=bd, valid=vd)
        else:
            o = avey_b(tail, z_tl=head, bias=bd, valid=vd)
        ev_cmp[k].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[k])
            out_host[k].copy_(o, non_blocking=True)  # stream order protects out_host[k]
            o.record_stream(s_out)

    def e2e_run(n):
        first = torch.cuda.Event(enable_timing=True)
        last = torch.cuda.Event(enable_timing=True)
        first.record(s_cmp)
        s_in.wait_stream(s_cmp)
        s_out.wait_stream(s_cmp)
        for i in range(n):
            e2e_step(i)
        s_cmp.wait_stream(s_in)
        s_cmp.wait_stream(s_out)
        last.record(s_cmp)
        return first, last

    e2e_run(3)
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = e2e_run(e2e_steps)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e2e_steps, device=dev)
    # The last step's output, read back through the pipeline, is the timed region's result.
    assert torch.isfinite(out_host[(e2e_steps - 1) % 2].float()).all()
    e2e_value = tokens_per_step / (e2e_ms / 1e3)

    # The copy ceiling of that pipeline: the same pinned copies with no
    # compute, both directions at once on their streams, on every rank at once
    # (ranks share the host's memory and PCIe); and each direction alone.
    o_dev = [torch.empty(out_host[0].shape, dtype=out_host[0].dtype, device=dev) for _ in range(2)]

    def copy_run(n, h2d_on=True, d2h_on=True):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s_cmp)
        s_in.wait_stream(s_cmp)
        s_out.wait_stream(s_cmp)
        for i in range(n):
            k = i % 2
            if h2d_on:
                with torch.cuda.stream(s_in):
                    for dst, src in zip(dev_bufs[k], hosts):
                        if src is not None:
                            dst.copy_(src, non_blocking=True)
            if d2h_on:
                with torch.cuda.stream(s_out):
                    out_host[k].copy_(o_dev[k], non_blocking=True)
        s_cmp.wait_stream(s_in)
        s_cmp.wait_stream(s_out)
        b.record(s_cmp)
        return a, b

    copy_ms = {}
    for name, kw in (('both', {}), ('h2d', dict(d2h_on=False)), ('d2h', dict(h2d_on=False))):
        copy_run(2, **kw)
        torch.cuda.synchronize()
        barrier()
        a, b = copy_run(e2e_steps, **kw)
        torch.cuda.synchronize()
        barrier()
        copy_ms[name] = max_over_ranks(a.elapsed_time(b) / e2e_steps, device=dev)
    ceiling_ms = max(copy_ms['both'], ms_step)

    # Roofline of the dominant (only) kernel.
    nbytes, flops = algorithmic(cfg, batch, sets[0]['valid'])
    t_launch = ms_step / 1e3
    gbs = nbytes / t_launch / 1e9
    tflops = flops / t_launch / 1e12
    hbm_time = nbytes / (peaks['hbm_gbs'] * 1e9)
    tc_time = flops / (peaks['bf16_tflops'] * 1e12)
    bound = 'hbm' if hbm_time >= tc_time else 'tensor'
    traffic = None
    prof = ROOT / 'profiles' / 'traffic.json'
    if prof.exists():
        entry = json.loads(prof.read_text()).get(args.config, {})
        if entry.get('kernel') == kernel_name:
            traffic = entry.get('dram_bytes_per_launch')
    if bound == 'hbm':
        roof = {'bound': 'hbm', 'achieved': gbs, 'peak': peaks['hbm_gbs'], 'unit': 'GB/s',
                'frac': gbs / peaks['hbm_gbs']}
    else:
        roof = {'bound': 'tensor', 'achieved': tflops, 'peak': peaks['bf16_tflops'],
                'unit': 'TFLOP/s', 'frac': tflops / peaks['bf16_tflops']}
    roof.update({'traffic': traffic, 'traffic_ratio': traffic / nbytes if traffic else None,
                 'kernel': kernel_name, 'peak_source': peaks['source'],
                 'algorithmic_bytes': nbytes, 'useful_flops': flops,
                 'hbm_frac': gbs / peaks['hbm_gbs'], 'tensor_frac': tflops / peaks['bf16_tflops'],
                 'tensor_tflops': tflops, 'binding_floor_us': 1e6 * max(hbm_time, tc_time),
                 'binding_frac': max(hbm_time, tc_time) / t_launch})

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        with all_host_threads():
            cpu_value, cpu_steps, cpu_busy = time_cpu_port(cfg, seconds=args.cpu_seconds, rows=1)
            cpu_cores = cpu_threads()
        cpu = {'value': cpu_value, 'unit': UNIT, 'cores': cpu_cores, 'kind': 'port',
               'sample': f'{cpu_steps} runs of 1 batch row ({cfg["n"]} tokens) of {args.config}, '
                         f'{cpu_busy:.1f} s, fp32 NumPy port of avey_kernels/ops.py::_reference'}
        # The same port on one thread, for reference (a shorter sample).
        try:
            from threadpoolctl import threadpool_limits
            with threadpool_limits(limits=1):
                one_value, one_steps, one_busy = time_cpu_port(
                    cfg, seconds=max(1.0, args.cpu_seconds / 4), rows=1)
            cpu['single_thread'] = {'value': one_value, 'unit': UNIT, 'cores': 1,
                                    'sample': f'{one_steps} runs, {one_busy:.1f} s'}
        except Exception as exc:  # pragma: no cover - reported, not fatal
            cpu['single_thread'] = {'error': repr(exc)[:200]}

    if rank == 0:
        line = {
            'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms_step,
            'higher_is_better': True, 'scaling': cfg['scaling'], 'vs_baseline': None,
            'dtype': 'f32' if f32 else 'bf16', 'data': 'synthetic (seeded randn, BASELINE config shapes)',
            'config': {'workload': f'{args.config}: {cfg["desc"]}', 'context': cfg['n'],
                       'features': cfg['d'], 'batch_per_gpu': batch,
                       'global_batch': batch * world, 'parallelism': f'dp{world} (batch shards)',
                       'l2': (f'inputs rotate over {nsets} sets of '
                              f'{nsets * sets[0]["x"].numel() * sets[0]["x"].element_size() / 1e6:.0f}'
                              ' MB total' + (' > 126 MB L2' if nsets * sets[0]['x'].numel() *
                                             sets[0]['x'].element_size() > 126e6 else
                                             ' (fits in L2: a latency-bound config)')),
                       'timing': 'CUDA graphs replayed between CUDA events, max over ranks'},
            'e2e': {'value': e2e_value, 'unit': UNIT, 'h2d_bytes_per_step': h2d * world,
                    'd2h_bytes_per_step': d2h * world, 'ms_per_step': e2e_ms,
                    'pipelining': 'copy-in of step i+1, compute of step i and copy-out of step i-1 overlap (3 streams, 2 buffer sets)',
                    'api': f'avey_kernel_b200.{cfg["op"]} (pinned host buffers)',
                    'copy_ceiling': {
                        'how': 'the same pinned copies per step with no compute, max over ranks '
                               '(all ranks copying at once); ceiling = max(both directions, '
                               'device step)',
                        'ms_per_step_both': copy_ms['both'], 'ms_per_step_h2d': copy_ms['h2d'],
                        'ms_per_step_d2h': copy_ms['d2h'],
                        'h2d_gbs_per_rank': h2d / (copy_ms['h2d'] / 1e3) / 1e9,
                        'd2h_gbs_per_rank': d2h / (copy_ms['d2h'] / 1e3) / 1e9,
                        'value': tokens_per_step / (ceiling_ms / 1e3),
                        'e2e_frac_of_ceiling': ceiling_ms / e2e_ms}},
            'roofline': roof,
            'cpu_baseline': cpu,
            'clocks': clocks.summary(),
            'gpu_launches': gpu_launches * world,
            'verify': {'max_norm_rel_err_vs_oracle': verify_err, 'rows_per_rank': 2,
                       'tolerance': 1e-4 if f32 else 2e-2},
            'wall_s': time.perf_counter() - t0,
        }
        print(json.dumps(line), flush=True)
    del graphs, keep
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_triton(args, cfg):
    """The reference's GPU path (Triton) on this GPU, for comparison only."""
    world, rank, _ = rank_env()
    if rank != 0:
        return 0
    ref_dir = ROOT / 'baseline' / '_ref'
    try:
        sys.path.insert(0, str(ref_dir))
        from avey_kernels import ops as ref_ops
    except Exception as e:  # not installed on this box
        print(json.dumps({'impl': 'triton', 'unavailable': f'reference not importable from '
                                                           f'baseline/_ref: {e}'}), flush=True)
        return 0
    import torch
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    batch = shard_batch(cfg, world)
    d = cfg['d']
    nsets = 3
    sets = [make_inputs(cfg, batch, seed=s, device=dev) for s in range(nsets)]
    kw = dict(backend='triton', output_tile=args.triton_tile, autotune=args.triton_autotune)

    def call(s):
        t = sets[s]
        head, tail = t['x'][..., :d], t['x'][..., d:]
        if cfg['op'] == 'avey':
            return ref_ops.avey(tail, t['w'], z_tl=head, bias=t['bias'], valid=t['valid'], **kw)
        return ref_ops.avey_b(tail, z_tl=head, bias=t['bias'], valid=t['valid'], **kw)

    t0 = time.perf_counter()
    y = call(0)
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    # Parity of this run against the oracle on two rows (sanity of the baseline).
    import numpy as np
    import oracle
    t = sets[0]
    err = 0.0
    for r in sorted({0, batch - 1}):
        x = t['x'][r:r + 1].float().cpu().numpy()
        okw = dict(z_tl=x[..., :d], bias=t['bias'].float().cpu().numpy() if t['bias'] is not None else None,
                   valid=t['valid'][r:r + 1].cpu().numpy() if t['valid'] is not None else None)
        ref = (oracle.avey(x[..., d:], t['w'].float().cpu().numpy(), **okw) if cfg['op'] == 'avey'
               else oracle.avey_b(x[..., d:], **okw))
        got = y[r:r + 1].float().cpu().numpy()
        err = max(err, float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30)))
    for i in range(max(args.warmup, 3)):
        call(i % nsets)
    torch.cuda.synchronize()
    steps = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record()
        for i in range(steps):
            call(i % nsets)
        end.record()
        torch.cuda.synchronize()
    ms_step = start.elapsed_time(end) / steps
    value = batch * cfg['n'] / (ms_step / 1e3)
    line = {
        'impl': 'triton', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': 1,
        'steps': steps, 'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True,
        'dtype': 'bf16 inputs, fp32 arithmetic (tf32x3 MMA)', 'data': 'synthetic',
        'config': {'workload': f'{args.config}: {cfg["desc"]}', 'context': cfg['n'],
                   'features': cfg['d'], 'batch_per_gpu': batch, 'output_tile': args.triton_tile,
                   'autotune': args.triton_autotune,
                   'timing': 'eager calls between CUDA events (pre-pass, copies and kernel)'},
        'first_call_s': compile_s, 'clocks': clocks.summary(),
        'verify': {'max_norm_rel_err_vs_oracle': err, 'rows': 2},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_train(args, cfg):
    """Forward + backward on one GPU: ours (native) or the reference's autograd."""
    world, rank, _ = rank_env()
    if rank != 0:
        return 0
    import torch
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    batch = shard_batch(cfg, world)
    d, n = cfg['d'], cfg['n']
    if args.impl == 'reference':
        try:
            sys.path.insert(0, str(ROOT / 'baseline' / '_ref'))
            from avey_kernels import ops as api
        except Exception as e:
            print(json.dumps({'impl': 'reference', 'pass': 'train', 'unavailable':
                              f'reference not importable from baseline/_ref: {e}'}), flush=True)
            return 0
        kw = dict(backend='torch')
    else:
        import avey_kernel_b200 as api
        from avey_kernel_b200 import _native
        kw = dict(backend='cuda')
    nsets = 2
    sets = []
    for s_ in range(nsets):
        t = make_inputs(cfg, batch, seed=s_, device=dev)
        g = torch.Generator().manual_seed(100 + s_)
        t['gout'] = torch.randn(batch, n, d, generator=g).to(torch.bfloat16).to(dev)
        t['x'].requires_grad_(True)
        if t['w'] is not None:
            t['w'].requires_grad_(True)
        if t['bias'] is not None:
            t['bias'].requires_grad_(True)
        sets.append(t)

    def step(i):
        t = sets[i % nsets]
        head, tail = t['x'][..., :d], t['x'][..., d:]
        if cfg['op'] == 'avey':
            out = api.avey(tail, t['w'], z_tl=head, bias=t['bias'], valid=t['valid'], **kw)
        else:
            out = api.avey_b(tail, z_tl=head, bias=t['bias'], valid=t['valid'], **kw)
        leaves = [x for x in (t['x'], t['w'], t['bias']) if x is not None]
        return torch.autograd.grad(out, leaves, t['gout'])

    grads = step(0)
    torch.cuda.synchronize()
    # Parity of the x gradient on one batch row against the gradient oracle.
    import numpy as np
    from oracle.backward import contextualize_backward
    t = sets[0]
    x = t['x'][:1].detach().float().cpu().numpy()
    okw = dict(eps=1e-6, norm_eps=1e-12, causal=cfg['op'] == 'avey',
               normalize=cfg['op'] == 'avey_b', activation='identity')
    w_np = t['w'].detach().float().cpu().numpy() if t['w'] is not None else None
    b_np = t['bias'].detach().float().cpu().numpy() if t['bias'] is not None else None
    v_np = t['valid'][:1].cpu().numpy() if t['valid'] is not None else None
    gz, _, gzl, _ = contextualize_backward(x[..., d:], w_np, x[..., :d], b_np, v_np,
                                           t['gout'][:1].float().cpu().numpy(), **okw)
    ref = np.concatenate([gzl, gz], axis=-1)
    got = grads[0][:1].float().cpu().numpy()
    err = float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()

    def timed(run):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.steps):
            run(i)
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / args.steps

    launches0 = _native.launch_count() if args.impl != 'reference' else None
    eager_ms = timed(step)
    launches = _native.launch_count() - launches0 if launches0 is not None else None
    # The same steps replayed from CUDA graphs (one per input set), which
    # takes the host's per-op dispatch cost out of the device timeline.
    graphs, graph_error = [], None
    try:
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for k in range(nsets):
                step(k)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        for k in range(nsets):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step(k)
            graphs.append(gr)
        for gr in graphs:
            gr.replay()
        torch.cuda.synchronize()
    except Exception as exc:  # a path that cannot be captured keeps the eager number
        graphs, graph_error = [], f'{type(exc).__name__}: {exc}'[:200]
    with ClockSampler(dev.index) as clocks:
        ms_step = timed(lambda i: graphs[i % nsets].replay()) if graphs else timed(step)
    # Dense GEMM work of the native backward (five [N,N]x[N,d'] products per
    # row) plus the forward's useful work.
    _, fwd_flops = algorithmic(cfg, batch, t['valid'])
    bwd_gemm_flops = 5 * 2 * batch * n * n * d
    line = {
        'impl': args.impl, 'pass': 'train', 'metric': 'contextualizer fwd+bwd tokens/s',
        'value': batch * n / (ms_step / 1e3), 'unit': 'tokens/s', 'n_gpus': 1,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms_step,
        'higher_is_better': True, 'dtype': 'bf16' if args.impl != 'reference' else
        'bf16 inputs, fp32 arithmetic', 'data': 'synthetic',
        'config': {'workload': f'{args.config}: {cfg["desc"]}', 'batch_per_gpu': batch,
                   'grads': 'x (head and tail), W, bias',
                   'timing': ('forward + torch.autograd.grad captured in CUDA graphs, replayed '
                              if graphs else 'eager forward + torch.autograd.grad ') +
                             'between CUDA events; every step streams > 1 GB, larger than L2'},
        'eager_ms_per_step': eager_ms,
        'tflops_fwd_useful_plus_bwd_gemm': (fwd_flops + bwd_gemm_flops) / (ms_step / 1e3) / 1e12,
        'clocks': clocks.summary(),
        'verify': {'grad_x_max_norm_rel_err_vs_oracle': err, 'rows': 1},
    }
    if graph_error:
        line['graph_capture_error'] = graph_error
    if launches is not None:
        line['gpu_launches'] = launches
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=3000)
    ap.add_argument('--warmup', type=int, default=10)
    ap.add_argument('--impl', choices=('ours', 'reference', 'triton'), default='ours')
    ap.add_argument('--triton-tile', type=int, choices=(32, 64, 128), default=128)
    ap.add_argument('--triton-autotune', action='store_true')
    ap.add_argument('--config', choices=tuple(CONFIGS), default='c2')
    ap.add_argument('--cpu-seconds', type=float, default=10.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--pass', dest='pass_', choices=('fwd', 'train'), default='fwd')
    args = ap.parse_args()
    if args.steps < 1 or args.warmup < 0:
        ap.error('--steps must be >= 1 and --warmup >= 0')
    world, _, _ = rank_env()
    if world != args.gpus and args.impl == 'ours':
        ap.error(f'--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun')
    cfg = CONFIGS[args.config]
    if args.pass_ == 'train':
        return run_train(args, cfg)
    if args.impl == 'reference':
        return run_reference(args, cfg)
    if args.impl == 'triton':
        return run_triton(args, cfg)
    return run_ours(args, cfg)


if __name__ == '__main__':
    sys.exit(main())
