"""Benchmark of the semantic-ID-constrained beam path: ms per user and users/sec.

One step = one user request (batch 1, 50 beams): prefill of the user's
history into the shared prefix, four decode forwards, five step tails
(double log-softmax over the full vocabulary, trie mask, beam top-k, parent
gather).  Default workload: the Qwen2.5-1.5B-shaped FP32 model, 3,500-item
catalog, prompts of 150-350 tokens (synthetic, seeded).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank drives one GPU; users are dealt round-robin (weak
scaling: every rank serves K users) and no collective runs on the per-step
path - a barrier and max-reduction of the timings bracket the timed region.

* ``value``: users/s over all ranks with the prompts already in HBM, timed
  with CUDA events on the launching stream (requests queued back to back);
  median/p95 are per-user device times.
* ``e2e``: the same through the public host API (``BeamEngine.generate``: pinned
  H2D of the prompt, D2H of the ranked result, sync-to-sync per user, the
  reference's timing span ``benchmark_inference.py:230-232``).
* ``roofline``: the decode projection GEMMs (dominant kernel), algorithmic
  weight bytes per pass / device time, against the measured HBM copy peak.
* ``concurrent`` (``--sessions S``, default 2): the same users served by S
  independent sessions per GPU on separate streams (each request still batch
  1), so one user's GEMMs fill another's small kernels and launch gaps;
  ``value`` stays the sequential figure the reference's protocol measures.
* ``--impl reference``: the reference algorithm on the host cores (the CPU
  oracle port of HF generate + the reference's processor), rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = 'median/p95 ms per user (batch 1, beam 50) and users/sec at 1/2/4/8 B200'


def percentile(values, q):
    """Linear interpolation at (n-1)*q, as ``benchmark.py:64-68``."""
    ordered = sorted(values)
    idx = (len(ordered) - 1) * q
    lo, hi = int(idx), min(int(idx) + 1, len(ordered) - 1)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (idx - lo)


# DRAM bytes of one decode GEMM pass (every projection at M = 50 plus the LM
# head): ncu dram__bytes_read.sum + dram__bytes_write.sum of a one-layer cut
# (`--mode profile-gemms --rows 50 --layers 1`), the layer's share scaled by
# the layer count.  Workloads without a capture report null.
GEMM_PASS_TRAFFIC = {'qwen1.5b-fp32': 6.317e9, 'qwen1.5b-bf16': 3.169e9}
GEMM_PASS_TRAFFIC_TF32 = {'qwen1.5b-fp32': 6.426e9}   # the 3xTF32 kernels (RTR_GEMM=tf32)


def measured_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return d['hbm_gbs'], 'measured'
    return 6650.0, 'fallback'


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""
    FIELDS = ('uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '200'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [x.strip() for x in line.split(',')]
            if len(parts) < 9 or (self.uuid and self.uuid not in parts[0]):
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == 'active':
                    reasons.add(name)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled'], 'samples': 0}
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(smax), 'reasons': sorted(reasons),
                'samples': len(sm)}


def physical_cores():
    """Physical cores this process may run on (``/proc/cpuinfo`` core ids of the
    allowed logical CPUs); logical CPUs where the core ids are not readable."""
    try:
        allowed = os.sched_getaffinity(0)
    except AttributeError:
        allowed = set(range(os.cpu_count() or 1))
    cores, cpu, phys = set(), None, None
    try:
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            key, _, val = (x.strip() for x in line.partition(':'))
            if key == 'processor':
                cpu, phys = int(val), None
            elif key == 'physical id':
                phys = int(val)
            elif key == 'core id' and cpu in allowed:
                cores.add((phys, int(val)))
    except (OSError, ValueError):
        cores = set()
    return len(cores) or len(allowed)


def bench_config(args, wl, world, beams=50):
    """The ``config`` object of both arms' JSON lines."""
    cfg = wl.model
    return {'workload': args.workload, 'model': cfg.name, 'beams': beams, 'items': wl.items,
            'prompt_tokens': [wl.prompt_min, wl.prompt_max], 'users_per_rank': args.steps,
            'parallelism': f'replicas{world}', 'partition': 'users round-robin, no per-step collective',
            'l2': f'inputs larger than L2: the {gemm_weight_bytes(cfg) / 1e9:.1f} GB of weights stream from HBM '
                  f'every forward'}


def dist_env():
    return int(os.environ.get('RANK', 0)), int(os.environ.get('LOCAL_RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))


def build_workload(name, n_users):
    from rapidtinyrec_b200 import configs, workload
    wl = configs.workload(name)
    items = workload.catalog_items(wl)
    cons = workload.constraint_dict(wl.model, items)
    users = workload.users(wl, items, count=min(n_users, wl.users))
    while len(users) < n_users:  # cycle the cohort if more steps than users are asked
        users = users + users[:n_users - len(users)]
    return wl, items, cons, users


def gemm_weight_bytes(cfg):
    b = 4 if cfg.dtype == 'fp32' else 2
    layer = cfg.qkv_dim * cfg.hidden + cfg.qkv_dim + cfg.hidden * cfg.q_dim + 3 * cfg.hidden * cfg.intermediate
    return b * (cfg.layers * layer + cfg.vocab * cfg.hidden)


def cpu_oracle_time(cfg, weights_cpu, cons, users, budget_s, threads):
    """Time the CPU port of the reference path on a bounded sample of users."""
    import torch
    from oracle.beam_cpu import beam_search
    from oracle.qwen2_cpu import Qwen2Oracle
    torch.set_num_threads(threads)
    model = Qwen2Oracle(cfg, weights_cpu, dtype=torch.bfloat16 if cfg.dtype == 'bf16' else torch.float32)
    times = []
    t_start = time.perf_counter()
    for u in users:
        t0 = time.perf_counter()
        beam_search(model, u.prompt_token_ids, cons, cfg.eos)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return times


def decode_step_roofline(engine, cfg, users, ids_dev, stream, peak):
    """Device time of decode steps 1-4 inside requests (CUDA events around each
    step on the session's stream) against the bytes a step must move: every
    weight once (layers, LM head, final norm) plus the K/V it reads (the shared
    prefix and the beams' suffix rows) and writes (50 new rows)."""
    import torch
    b = 4 if cfg.dtype == 'fp32' else 2
    kv_token = 2 * cfg.kv_heads * cfg.head_dim * cfg.layers * b
    times, nbytes = [], []
    for i, u in enumerate(users):
        L = u.prompt_tokens
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        engine._check(engine.lib.rtr_prefill(engine.handle, ids_dev[i].data_ptr(), L, 1))
        ev[0].record(stream)
        for t in range(1, 5):
            engine.decode_step(t)
            ev[t].record(stream)
        engine.read_results()
        torch.cuda.synchronize()
        for t in range(1, 5):
            times.append(ev[t - 1].elapsed_time(ev[t]))
            nbytes.append(cfg.weight_bytes_per_step() + kv_token * (L + engine.beams * (t - 1)) +
                          kv_token * engine.beams)
    ms = statistics.median(times)
    byt = statistics.median(nbytes)
    achieved = byt / (ms / 1000.0) / 1e9
    return {'bound': 'hbm', 'ms_per_step': round(ms, 4), 'bytes_per_step': int(byt), 'achieved': round(achieved, 1),
            'peak': peak, 'unit': 'GB/s', 'frac': round(achieved / peak, 4),
            'steps_timed': len(times), 'note': 'median decode step 1-4 inside requests (weights + prefix/suffix K/V '
                                               'read + new K/V written) / CUDA-event step time'}


def run_reference(args):
    """The reference algorithm on the host cores: the CPU oracle port of HF beam
    search + the reference's processor + folded SDPA, with weights made by the
    numpy restatement of the synthetic filler (no library of this repository is
    loaded on this arm)."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    import torch
    from rapidtinyrec_b200 import workload as wk
    threads = physical_cores()
    wl, _, cons, users = build_workload(args.workload, args.warmup + args.steps)
    cfg = wl.model
    weights = wk.synth_weights(cfg, seed=wl.weight_seed, device='cpu', backend='numpy', threads=threads)
    warm = cpu_oracle_time(cfg, weights, cons, users[:min(args.warmup, 3)], 1e9, threads)
    # bound the run: every step is one full request; cap the count to ~150 s of CPU work
    per = statistics.median(warm) if warm else 1.0
    k = max(1, min(args.steps, int(150.0 / max(per, 1e-3))))
    times = cpu_oracle_time(cfg, weights, cons, users[args.warmup:args.warmup + k], 1e9, threads)
    total = sum(times)
    value = len(times) / total
    line = {'metric': METRIC, 'impl': 'reference', 'value': round(value, 4), 'unit': 'users/s',
            'n_gpus': world, 'steps': len(times), 'warmup': len(warm), 'ms_per_step': round(1000 * total / len(times), 2),
            'median_ms': round(1000 * statistics.median(times), 2), 'p95_ms': round(1000 * percentile(times, 0.95), 2),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'f32' if cfg.dtype == 'fp32' else 'bf16',
            'data': 'synthetic', 'config': bench_config(args, wl, world),
            'cpu_baseline': {'value': round(value, 4), 'unit': 'users/s', 'cores': threads, 'kind': 'port',
                             'sample': f'{len(times)} users of {args.workload} (of {args.steps} requested), full '
                                       f'request each (CPU oracle port of HF beam search + '
                                       f'GpuSidConstrainedLogitsProcessor + folded SDPA), torch on {threads} '
                                       f'threads = physical cores'},
            'e2e': {'value': round(value, 4), 'unit': 'users/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def rank_users(all_users, rank, world):
    """This rank's users: dealt round-robin (rank, rank + world, ...); the ranks
    share nothing on the per-step path."""
    return all_users[rank::world]


def combine_ranks(total_ms, e2e_total, per_user, e2e_lat, world, device):
    """The job's timing from every rank's own, outside the timed region: the max
    of the ranks' timed spans (the job ends with its slowest rank) and every
    rank's per-user latencies, rank after rank.  One rank returns its own."""
    if world == 1:
        return total_ms, e2e_total, per_user, e2e_lat
    import torch
    import torch.distributed as dist
    t = torch.tensor([total_ms, e2e_total], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    lat = torch.tensor(per_user, dtype=torch.float64, device=device)
    gathered = [torch.empty_like(lat) for _ in range(world)]
    dist.all_gather(gathered, lat)
    el = torch.tensor(e2e_lat, dtype=torch.float64, device=device)
    g2 = [torch.empty_like(el) for _ in range(world)]
    dist.all_gather(g2, el)
    return (float(t[0]), float(t[1]), [float(x) for g in gathered for x in g.tolist()],
            [float(x) for g in g2 for x in g.tolist()])


def run_ours(args):
    import torch
    import torch.distributed as dist
    from rapidtinyrec_b200 import workload as wk
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)

    per_rank = args.warmup + args.steps
    wl, items, cons, all_users = build_workload(args.workload, per_rank * world)
    users = rank_users(all_users, rank, world)
    cfg = wl.model
    max_prefix = max(wl.prompt_max, max(u.prompt_tokens for u in users))
    weights = wk.synth_weights(cfg, seed=wl.weight_seed, device=f'cuda:{local}')
    tables = GpuSidConstraintTables(cons, cfg.root, cfg.newline, cfg.eos)
    engine = BeamEngine(cfg, weights, tables, max_prefix=max_prefix, device=local, max_users=max(1, args.batch))
    # extra independent sessions for the concurrent-serving measurement
    extra = [BeamEngine(cfg, weights, tables, max_prefix=max_prefix, device=local)
             for _ in range(max(0, args.sessions - 1))]
    weights_cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        weights_cpu = {k: v.cpu() for k, v in weights.items()}
    del weights
    torch.cuda.empty_cache()
    stream = torch.cuda.Stream(device=dev)
    engine.set_stream(stream)

    ids_dev = [torch.tensor(u.prompt_token_ids, dtype=torch.int32, device=dev) for u in users]
    ids_host = [torch.tensor(u.prompt_token_ids, dtype=torch.int32).numpy() for u in users]
    torch.cuda.synchronize(dev)

    # warm-up (graph capture happens on the first request)
    for i in range(args.warmup):
        engine.launch_device(ids_dev[i], users[i].prompt_tokens)
        engine.wait()

    def barrier():
        if world > 1:
            dist.barrier()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass

    # ---- device-resident timed region
    timed = range(args.warmup, args.warmup + args.steps)
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    launches_before = engine.report()['kernel_launches']
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(uuid) as clocks:
        events[0].record(stream)
        for j, i in enumerate(timed):
            engine.launch_device(ids_dev[i], users[i].prompt_tokens)
            events[j + 1].record(stream)
        engine.wait()
        torch.cuda.synchronize(dev)
    barrier()
    launches = engine.report()['kernel_launches'] - launches_before
    per_user = [events[j].elapsed_time(events[j + 1]) for j in range(args.steps)]
    total_ms = events[0].elapsed_time(events[-1])

    # ---- end-to-end through the host API
    e2e_lat = []
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in timed:
        t = time.perf_counter()
        engine.generate_raw(ids_host[i])
        e2e_lat.append(time.perf_counter() - t)
    e2e_total = time.perf_counter() - t0
    barrier()
    rep = engine.report()

    # ---- concurrent serving: S independent sessions on their own streams,
    # batch-1 requests dealt round-robin (device-resident prompts)
    concurrent = None
    if extra:
        sessions = [(engine, stream)] + [(e, torch.cuda.Stream(device=dev)) for e in extra]
        for e, st in sessions[1:]:
            e.set_stream(st)
        for k, (e, _) in enumerate(sessions):  # warm-up (graph capture)
            e.launch_device(ids_dev[k % len(ids_dev)], users[k % len(users)].prompt_tokens)
        for e, _ in sessions:
            e.wait()
        torch.cuda.synchronize(dev)
        start = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _, st in sessions[1:]:
            st.wait_event(start)
        for j, i in enumerate(timed):
            e, _ = sessions[j % len(sessions)]
            if j >= len(sessions):
                e.wait()  # the session's previous request leaves its slot
            e.launch_device(ids_dev[i], users[i].prompt_tokens)
        ends = []
        for e, st in sessions:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(st)
            ends.append(ev)
        for e, _ in sessions:
            e.wait()
        torch.cuda.synchronize(dev)
        conc_ms = max(start.elapsed_time(ev) for ev in ends)
        if world > 1:
            t = torch.tensor([conc_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            conc_ms = float(t[0])
        concurrent = {'sessions': len(sessions), 'value': round(args.steps * world / (conc_ms / 1000.0), 3),
                      'unit': 'users/s', 'ms_per_step': round(conc_ms / args.steps, 3),
                      'note': 'independent sessions (one weight copy each) on separate streams, batch-1 requests '
                              'dealt round-robin, prompts in HBM; CUDA events, max over ranks'}
        for e in extra:
            e.close()

    # ---- batched serving: groups of U users share each decode step (one session,
    # one weight copy; every projection GEMM at U x 50 rows)
    batched = None
    if args.batch > 1:
        U = args.batch
        groups = [list(range(args.warmup + k, min(args.warmup + k + U, args.warmup + args.steps)))
                  for k in range(0, args.steps, U)]
        groups = [g for g in groups if len(g) == U] or groups[:1]
        for _ in range(2):  # warm-up (graph capture for U users)
            engine.launch_batch_device([ids_dev[i] for i in range(U)], [users[i].prompt_tokens for i in range(U)])
            engine.wait_batch()
        torch.cuda.synchronize(dev)
        bev = [torch.cuda.Event(enable_timing=True) for _ in range(len(groups) + 1)]
        barrier()
        torch.cuda.synchronize(dev)
        bev[0].record(stream)
        for k, g in enumerate(groups):  # queued back to back, like the batch-1 timed region
            engine.launch_batch_device([ids_dev[i] for i in g], [users[i].prompt_tokens for i in g])
            bev[k + 1].record(stream)
        engine.wait_batch()
        torch.cuda.synchronize(dev)
        b_ms = bev[0].elapsed_time(bev[-1])
        n_batched = sum(len(g) for g in groups)
        if world > 1:
            t = torch.tensor([b_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            b_ms = float(t[0])
        batched = {'users_per_batch': U, 'value': round(n_batched * world / (b_ms / 1000.0), 3), 'unit': 'users/s',
                   'ms_per_batch': round(b_ms / len(groups), 3),
                   'note': 'one session, U users per request: each user prefilled on its own, then decode steps '
                           '1-4 for all U users in one graph (GEMMs at U x 50 rows); prompts in HBM; CUDA events, '
                           'max over ranks'}

    # ---- roofline of the dominant kernel: the decode projection GEMMs (M = beams)
    gemm_ms = engine.profile_gemms(engine.beams, reps=5)
    step_roof = decode_step_roofline(engine, cfg, [users[i] for i in timed][:6], [ids_dev[i] for i in timed][:6],
                                     stream, measured_peaks()[0])
    gemm_bytes = gemm_weight_bytes(cfg)
    peak, peak_kind = measured_peaks()

    total_ms, e2e_total, per_user, e2e_lat = combine_ranks(total_ms, e2e_total, per_user, e2e_lat, world, dev)

    cpu = None
    if weights_cpu is not None:
        threads = physical_cores()
        times = cpu_oracle_time(cfg, weights_cpu, cons, users[args.warmup:], args.cpu_budget, threads)
        cpu = {'value': round(len(times) / sum(times), 5), 'unit': 'users/s', 'cores': threads, 'kind': 'port',
               'sample': f'{len(times)} users of {args.workload} (full request each) through the CPU oracle port '
                         f'of HF beam search + GpuSidConstrainedLogitsProcessor + folded SDPA, torch on {threads} '
                         f'threads = physical cores, median {1000 * statistics.median(times):.0f} ms/user'}

    if rank == 0:
        n_users = args.steps * world
        value = n_users / (total_ms / 1000.0)
        achieved = gemm_bytes / (gemm_ms / 1000.0) / 1e9
        ck = clocks.summary()
        gemm_flops = 2.0 * engine.beams * gemm_bytes / (4 if cfg.dtype == 'fp32' else 2)
        if cfg.dtype == 'bf16':
            gemm_kernel = 'gemm_bf16_kernel (tcgen05 kind::f16'
        else:
            gemm_kernel = {2: 'gemm_f16x2_kernel (tcgen05 fp16 pairs', 1: 'gemm_tc_kernel (tcgen05 3xTF32'}.get(
                rep['tensor_core_gemm'], 'gemm_f32_kernel (FFMA')
        gemm_kernel += f', decode projections + LM head, M={engine.beams})'
        line = {
            'metric': METRIC, 'value': round(value, 3), 'unit': 'users/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': round(total_ms / args.steps, 3),
            'median_ms': round(statistics.median(per_user), 3), 'p95_ms': round(percentile(per_user, 0.95), 3),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'f32' if cfg.dtype == 'fp32' else 'bf16', 'data': 'synthetic',
            'config': bench_config(args, wl, world, engine.beams),
            'e2e': {'value': round(n_users / e2e_total, 3), 'unit': 'users/s',
                    'median_ms': round(1000 * statistics.median(e2e_lat), 3),
                    'p95_ms': round(1000 * percentile(e2e_lat, 0.95), 3),
                    'h2d_bytes_per_step': rep['h2d_bytes_per_request'],
                    'd2h_bytes_per_step': rep['d2h_bytes_per_request'],
                    'timing': 'host wall clock, sync to sync per user'},
            'roofline': {'bound': 'hbm', 'kernel': gemm_kernel,
                         'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
                         'frac': round(achieved / peak, 4), 'peak_source': peak_kind,
                         'traffic': (GEMM_PASS_TRAFFIC_TF32 if cfg.dtype == 'fp32' and rep['tensor_core_gemm'] == 1
                                     else GEMM_PASS_TRAFFIC).get(args.workload), 'traffic_source':
                             'ncu dram__bytes_read+write of a one-layer cut, layer share x layers + LM head'
                             if args.workload in GEMM_PASS_TRAFFIC
                             else None,
                         'bytes_per_pass': gemm_bytes, 'ms_per_pass': round(gemm_ms, 4),
                         'gemm_tflops': round(gemm_flops / (gemm_ms / 1000.0) / 1e12, 2)},
            'decode_step_roofline': step_roof,
            'gpu_launches': int(launches),
            'concurrent': concurrent,
            'batched': batched,
            'launches_per_user': rep['launches_per_request'],
            'clocks': ck,
        }
        if cpu is not None:
            line['cpu_baseline'] = cpu
        print(json.dumps(line), flush=True)
    engine.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile(args):
    """Small, self-contained launch sequences for ncu captures (one GPU).

    profile-request: one warm-up request, then one request bracketed by
      cudaProfilerStart/Stop (use ncu --profile-from-start off).
    profile-gemms: a model cut to --layers layers; every projection GEMM of one
      forward over --rows rows runs twice (warm-up pass + one timed pass).
    profile-phases: device time of each phase of a request (CUDA events on the
      session's stream): prefill + step 0 and each decode step through the
      per-step entry points, the whole request through the captured graph, and
      the GEMM passes at the decode and prefill row counts.
    """
    import dataclasses
    import torch
    from rapidtinyrec_b200 import workload as wk
    from rapidtinyrec_b200.constraints import GpuSidConstraintTables
    from rapidtinyrec_b200.engine import BeamEngine
    wl, _, cons, users = build_workload(args.workload, max(2, args.users))
    cfg = wl.model if args.layers is None else dataclasses.replace(wl.model, layers=args.layers)
    weights = wk.synth_weights(cfg, seed=wl.weight_seed, device='cuda')
    engine = BeamEngine(cfg, weights, GpuSidConstraintTables(cons, cfg.root, cfg.newline, cfg.eos),
                        max_prefix=max(wl.prompt_max, args.rows))
    del weights
    torch.cuda.empty_cache()
    if args.mode == 'profile-request':
        engine.generate(users[0].prompt_token_ids)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        t0 = time.perf_counter()
        engine.generate(users[1].prompt_token_ids)
        torch.cuda.profiler.stop()
        print(json.dumps({'mode': args.mode, 'prompt_tokens': users[1].prompt_tokens,
                          'wall_ms': 1000 * (time.perf_counter() - t0), 'report': engine.report()}))
    elif args.mode == 'profile-phases':
        st = torch.cuda.Stream()
        engine.set_stream(st)
        dev_ids = [torch.tensor(u.prompt_token_ids, dtype=torch.int32, device='cuda') for u in users]
        for u in users[:3]:  # warm-up: graph capture and first launches
            engine.generate(u.prompt_token_ids)
        phases = {'prefill_and_step0': [], 'step1': [], 'step2': [], 'step3': [], 'step4': [], 'request_graph': []}
        for i, u in enumerate(users):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
            torch.cuda.synchronize()
            ev[0].record(st)
            engine._check(engine.lib.rtr_prefill(engine.handle, dev_ids[i].data_ptr(), u.prompt_tokens, 1))
            ev[1].record(st)
            for t in range(1, 5):
                engine.decode_step(t)
                ev[t + 1].record(st)
            engine.read_results()
            ev[6].record(st)
            engine.launch_device(dev_ids[i], u.prompt_tokens)
            ev[7].record(st)
            engine.wait()
            torch.cuda.synchronize()
            phases['prefill_and_step0'].append(ev[0].elapsed_time(ev[1]))
            for t in range(1, 5):
                phases[f'step{t}'].append(ev[t].elapsed_time(ev[t + 1]))
            phases['request_graph'].append(ev[6].elapsed_time(ev[7]))
        lengths = [u.prompt_tokens for u in users]
        med_len = int(statistics.median(lengths))
        print(json.dumps({'mode': args.mode, 'workload': args.workload, 'users': len(users),
                          'prompt_tokens_median': med_len,
                          'median_ms': {k: round(statistics.median(v), 4) for k, v in phases.items()},
                          'gemm_pass_ms': {'decode_rows50': round(engine.profile_gemms(engine.beams, reps=5), 4),
                                           f'prefill_rows{med_len}': round(engine.profile_gemms(med_len, reps=5), 4)}}))
    else:
        print(json.dumps({'mode': args.mode, 'rows': args.rows, 'layers': cfg.layers,
                          'ms_per_pass': engine.profile_gemms(args.rows, reps=1)}))
    engine.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--mode', choices=('bench', 'profile-request', 'profile-gemms', 'profile-phases'),
                    default='bench')
    ap.add_argument('--users', type=int, default=12, help='profile-phases: requests timed')
    ap.add_argument('--rows', type=int, default=50, help='profile-gemms: activation rows')
    ap.add_argument('--layers', type=int, default=None, help='profile modes: cut the model to this many layers')
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=40)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--workload', default='qwen1.5b-fp32')
    ap.add_argument('--cpu-budget', type=float, default=20.0, help='seconds of CPU-baseline work (rank 0, N=1)')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--batch', type=int, default=4,
                    help='users per batched request for the batched-serving measurement (1: skip)')
    ap.add_argument('--sessions', type=int, default=2,
                    help='also measure S concurrent sessions per GPU (1: sequential only)')
    args = ap.parse_args()
    if args.mode != 'bench':
        run_profile(args)
        return
    if args.warmup < 3:
        ap.error('--warmup must be >= 3')
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
