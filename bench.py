#!/usr/bin/env python3
"""Benchmark: teacher-forced window scoring of the Mamba-2 8B FP4-G16 / SQ3.25 model.

Workload: full 56-layer model (vocab 256000, released per-layer
layouts), random-init FP4 G16 weights and statics of the recorded shapes, a random-init
Resurface adapter (soft gate), 16 reset windows x (2048 targets + 1 overlap token) per
GPU, token ids Zipf(s=1.1) over the vocabulary.  One step = scoring all local windows
(forward over 16 x 2048 tokens, fused lm_head + cross entropy) plus the one NLL-sum
all-reduce across ranks.  `value` = scored tokens/s over all ranks with the windows
already resident on the device; `e2e` = the same through the public scoring API from
pinned host buffers (H2D of the windows, D2H of the per-window NLLs, every step).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
  python bench.py --case gemm|scan|decode|gemv|s16 [--layout L|all] [--layers N --vocab V] [--rows M]
                  --steps K   (one kernel on a small case, for timing and ncu)
  torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU, NCCL)
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'mamb2_8b_fp4_recall_sq3.25_b200'))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = 'scored tokens/s (8B, per-token SQ3.25 requant)'
UNIT = 'tokens/s'
WINDOWS_PER_GPU, SEQLEN, VOCAB, N_LAYER = 16, 2048, 256000, 56
FLOP_PER_TOKEN = 2 * (56 * (18560 * 4096 + 4096 * 8192) + 256000 * 4096)   # 14,369,685,504
DECODE_BYTES_B1 = 4_111_674_420
# per decode step: FP4 layers + lm_head + fp16 small tensors + statics; per sequence: state
# rows r+w + conv ring r+w + embedding row (the per-unit figures of the decode roofline)
DECODE_FIXED_BYTES, DECODE_PER_SEQ_BYTES = 4_054_786_868, 56_887_552
FLOP_PER_TOKEN_BACKBONE = 2 * 56 * (18560 * 4096 + 4096 * 8192)                 # prefill, no lm_head
# dram__bytes_read.sum + dram__bytes_write.sum of one in_proj GEMM launch (M=32768), from
# one ncu --set full capture of `python bench.py --case gemm --steps 2` on this build.
GEMM_TRAFFIC_BYTES = 1_620_000_000 + 1_200_000_000   # ncu dram__bytes_read + write, one in_proj launch


def peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d['hbm_gbs'], tf=d['bf16_tflops'], tf_sus=d['bf16_tflops_sustained'], src='measured')
    return dict(hbm=6650.0, tf=1590.0, tf_sus=1400.0, src='fallback')


def zipf_tokens(n, rng, s=1.1, vocab=VOCAB):
    k = np.arange(1, vocab + 1, dtype=np.float64)
    p = k ** -s
    p /= p.sum()
    return rng.choice(vocab, size=n, p=p).astype(np.int64)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.index), '--query-gpu=' + self.FIELDS,
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(',')])

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=['nvidia-smi unavailable'])
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=['no samples'])
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        load = [x for x in sm if x > 0.5 * max(sm)] or sm
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower().startswith('active')})
        return dict(sm_mhz=statistics.median(load), sm_max_mhz=float(rows[0][2]), reasons=reasons,
                    samples=len(rows), power_w_max=max(float(r[3]) for r in rows if r[3].replace('.', '').isdigit()))


def dist_init(n):
    rank, world, local = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1)), \
        int(os.environ.get('LOCAL_RANK', 0))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device('cuda', local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


# ------------------------------------------------------------------ CPU reference arm

_CPU_MODELS = {}


def cpu_sample(tokens=2048, layers=3, vocab_slice=32768, seed=0):
    """The CPU oracle port (oracle/) on a bounded slice of the workload: one window of
    `tokens` tokens through `layers` full-geometry layers plus the lm_head + CE over a
    `vocab_slice`-row slice of the vocabulary, all host threads.  Returns seconds per
    scored token extrapolated to 56 layers and the full 256000-row head.  The oracle model
    is built once per process and reused by later samples."""
    from oracle.pair import build_pair
    torch.set_num_threads(os.cpu_count())
    key = (layers, vocab_slice, seed)
    if key not in _CPU_MODELS:
        _CPU_MODELS[key] = build_pair(n_layer=layers, vocab=vocab_slice, seed=seed, adapter=True, device=None)[1]
    ora = _CPU_MODELS[key]
    rng = np.random.default_rng(seed)
    ids = zipf_tokens(tokens + 1, rng, vocab=vocab_slice)[None]
    ora.reset(1)
    t0 = time.perf_counter()
    hid = ora.backbone(ids[:, :-1])
    t1 = time.perf_counter()
    ora.nll(hid, ids[:, 1:])
    t2 = time.perf_counter()
    per_token = ((t1 - t0) * N_LAYER / layers + (t2 - t1) * VOCAB / vocab_slice) / tokens
    return per_token, dict(tokens=tokens, layers=layers, vocab_slice=vocab_slice, seconds=t2 - t0)


def workload_config(world, B=WINDOWS_PER_GPU, T=SEQLEN):
    """The workload description both arms report (the reference arm on the same config)."""
    return dict(workload='config4: 56-layer 8B scoring, FP4-G16 weights, SQ3.25 state, Resurface soft',
                windows_per_gpu=B, seq_len=T, global_batch=world * B, vocab=VOCAB,
                parallelism=f'dp{world} (window-sharded, one NLL all-reduce)', l2='inputs larger than L2')


def run_reference(args, rank, world):
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup_ref):
        cpu_sample(tokens=args.ref_tokens)
    info = None
    for _ in range(max(1, args.steps_ref)):
        per_tok, info = cpu_sample(tokens=args.ref_tokens)
        vals.append(1.0 / per_tok)
    v = statistics.median(vals)
    line = dict(metric=METRIC, value=v, unit=UNIT, n_gpus=args.gpus, steps=len(vals), warmup=args.warmup_ref,
                ms_per_step=None, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32',
                data='synthetic', impl='reference',
                config=workload_config(max(world, args.gpus)),
                cpu_baseline=dict(value=v, unit=UNIT, cores=os.cpu_count(), kind='port',
                                  sample=f"oracle port, 1 window x {info['tokens']} tokens through {info['layers']} "
                                         f"layers + lm_head/CE over a {info['vocab_slice']}-row vocab slice, "
                                         f"extrapolated to 56 layers and 256000 rows ({platform.processor() or 'cpu'})"),
                e2e=dict(value=v, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

def build_workload(rank, device):
    from sq325 import model as M, resurface as R
    from sq325.state import PredictorState
    t0 = time.time()
    model = M.synthetic_model(seed=4, n_layer=N_LAYER, vocab=VOCAB, device=device)
    model.adapter = R.random_bank(N_LAYER, seed=5, device=device)
    statics = M.synthetic_statics(M.RELEASED_LAYOUTS, seed=4, device=device)
    ex = PredictorState(model, *statics).install()
    rng = np.random.default_rng(1000 + rank)
    wins = zipf_tokens(WINDOWS_PER_GPU * (SEQLEN + 1), rng).reshape(WINDOWS_PER_GPU, SEQLEN + 1)
    torch.cuda.synchronize()
    return model, ex, wins, time.time() - t0


def launches_per_step(M_rows, n_layer=N_LAYER, vocab=VOCAB):
    lin = 1 if M_rows <= 64 else 2
    per_layer = 1 + lin + 1 + 1 + 1 + lin          # add_rmsnorm, in_proj, scan prep, scan, resurface+norm, out_proj
    score = 2 * ((vocab + 32767) // 32768) + 1     # per 32768-row chunk: decode + gemm; finalize
    return 1 + n_layer * per_layer + 1 + score     # embed, layers, norm_f, head


def time_gemm_kernel(model, rows, device, reps=5):
    """Dominant kernel: the tcgen05 in_proj GEMM at the workload's shape, CUDA events on
    the launching stream (the operand decode is excluded by decoding once up front)."""
    from sq325 import _lib
    w = model.layers[0].in_proj
    lib = _lib.load()
    stage = torch.empty((w.rows, w.cols), device=device, dtype=torch.float16)
    _lib.call('sq_fp4_decode', _lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
              w.rows, w.cols, _lib.ptr(stage), w.cols, _lib.stream_ptr())
    x = torch.randn(rows, w.cols, device=device).half()
    y = torch.empty(rows, w.rows, device=device, dtype=torch.float16)
    s = torch.cuda.current_stream()
    for _ in range(2):
        _lib.call('sq_gemm_f16', _lib.ptr(x), w.cols, _lib.ptr(stage), w.cols, _lib.ptr(y), w.rows, rows, w.rows,
                  w.cols, _lib.stream_ptr())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ts = []
    for _ in range(reps):
        ev[0].record(s)
        _lib.call('sq_gemm_f16', _lib.ptr(x), w.cols, _lib.ptr(stage), w.cols, _lib.ptr(y), w.rows, rows, w.rows,
                  w.cols, _lib.stream_ptr())
        ev[1].record(s)
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]) / 1e3)
    del lib
    return statistics.median(ts), 2.0 * rows * w.rows * w.cols


@torch.no_grad()
def run_case(args):
    """One kernel on a small case, for ncu captures (a few GB on the device, steps + 3
    launches).  Prints one JSON line with CUDA-event timings; not a bench line."""
    from sq325 import _lib, codec
    torch.cuda.set_device(0)
    gen = torch.Generator(device='cuda').manual_seed(0)
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if args.case == 'decode':                     # persistent batch-1 decode step on a shortened model
        from sq325 import model as M, resurface as R
        from sq325.state import PredictorState
        model = M.synthetic_model(seed=4, n_layer=args.layers, vocab=args.vocab, device='cuda')
        model.adapter = R.random_bank(args.layers, seed=5, device='cuda')
        statics = M.synthetic_statics(M.RELEASED_LAYOUTS[:args.layers], seed=4, device='cuda')
        ex = PredictorState(model, *statics).install()
        ex.reserve(64)
        prompt = torch.from_numpy(zipf_tokens(64, np.random.default_rng(3)) % args.vocab)[None].cuda()
        tok = ex.greedy(ex.backbone(prompt, reset=True)[:, -1]).clone()
        call = lambda: ex.decode_persistent(tok, 1)
        unit, work = 'us/token', 1.0
    elif args.case == 'gemm':                     # tcgen05 in_proj GEMM at the scoring shape
        M, N, K = 32768, 18560, 4096
        a = torch.randn(M, K, device='cuda', generator=gen).half()
        b = (torch.randn(N, K, device='cuda', generator=gen) * 0.02).half()
        c = torch.empty(M, N, device='cuda', dtype=torch.float16)
        call = lambda: _lib.call('sq_gemm_f16', _lib.ptr(a), K, _lib.ptr(b), K, _lib.ptr(c), N, M, N, K,
                                 _lib.stream_ptr())
        unit, work = 'TFLOP/s', 2.0 * M * N * K
    elif args.case == 'gemv':                     # FP4 skinny GEMM, in_proj shape at M = args.rows (config 2)
        from sq325 import fp4 as F
        w = F.synthetic(18560, 4096, gen, 'cuda')
        x = torch.randn(args.rows, 4096, device='cuda', generator=gen).half()
        call = lambda: F.linear(w, x)
        unit, work = 'GB/s', 18560 * 4096 * 9 / 16 + args.rows * (4096 + 18560) * 2
    elif args.case == 's16':                      # FP16-state control scan, 16 x 128 x 64 rows, 512 tokens
        from sq325 import state_codec as sc
        B, L, H, P, G = 16, 512, 128, 64, 8
        x = torch.randn(B, L, H, P, device='cuda', generator=gen).half()
        dt = (torch.randn(B, L, H, device='cuda', generator=gen) * 0.5).half()
        A = -(torch.rand(H, device='cuda', generator=gen) * 3 + 0.1)
        Bm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        Cm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        D = torch.randn(H, device='cuda', generator=gen).half()
        db = (torch.rand(H, device='cuda', generator=gen) * 3 - 4).half()
        st = sc.allocate_state(B, H, P, 128, 's16', 'cuda')
        call = lambda: sc.scan(x, dt, A, Bm, Cm, D, db, st)
        unit, work = 'us/token', float(L)
    elif args.case in ('sq3p25', 'ste'):          # packed sq3p25 scan / its STE backward, training geometry
        import ctypes
        from sq325 import state_codec as sc
        B, L, H, P, G, K = STE_GEOMETRY
        x = torch.randn(B, L, H, P, device='cuda', generator=gen).half()
        dt = (torch.randn(B, L, H, device='cuda', generator=gen) * 0.5).half()
        A = -(torch.rand(H, device='cuda', generator=gen) * 3 + 0.1)
        Bm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        Cm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        D = torch.randn(H, device='cuda', generator=gen).half()
        db = (torch.rand(H, device='cuda', generator=gen) * 3 - 4).half()
        perm = torch.stack([torch.randperm(128, device='cuda', generator=gen) for _ in range(G)]).to(torch.uint8)
        if args.case == 'sq3p25':
            st = sc.allocate_state(B, H, P, 128, 'sq3p25', 'cuda')
            call = lambda: sc.scan(x, dt, A, Bm, Cm, D, db, st, permutation=perm)
        else:
            dy = torch.randn(B, L, H, P, device='cuda', generator=gen).half()
            grads = [torch.empty(t.shape, device='cuda', dtype=torch.float32) for t in (x, dt, Bm, Cm)]
            nbytes = int(_lib.load().sq_ste_workspace(B, L, H, P, K))
            ws = torch.empty(nbytes, device='cuda', dtype=torch.uint8)
            sargs = sc.sq3p25_args(x, dt, A, Bm, Cm, D, db, perm)
            call = lambda: _lib.call('sq_ste_backward', ctypes.byref(sargs), K, dy.data_ptr(),
                                     *(g.data_ptr() for g in grads), ws.data_ptr(), nbytes, _lib.stream_ptr())
        unit, work = 'us/token', float(L)
    else:                                         # SQ3.25 scan: prep + chunk kernels, 16 x 128 x 64 rows
        B, L, H, P, G = 16, 512, 128, 64, 8
        spec = codec.layout_descriptor(args.layout)
        n8, n4, nz = spec['n8'], spec['n4'], spec['nzero']
        x = torch.randn(B, L, H, P, device='cuda', generator=gen).half()
        dt = (torch.randn(B, L, H, device='cuda', generator=gen) * 0.5).half()
        A = -(torch.rand(H, device='cuda', generator=gen) * 3 + 0.1)
        Bm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        Cm = torch.randn(B, L, G, 128, device='cuda', generator=gen).half()
        D = torch.randn(H, device='cuda', generator=gen).half()
        db = (torch.rand(H, device='cuda', generator=gen) * 3 - 4).half()
        perm = torch.stack([torch.randperm(128, device='cuda', generator=gen) for _ in range(G)]).to(torch.uint8)
        basis = torch.randn(G, nz, 2, device='cuda', generator=gen).half()
        ls = (torch.rand(G, 2, device='cuda', generator=gen) + 0.1).half()
        pred = (torch.randn(G, n8 + n4 + 2, nz, device='cuda', generator=gen) / np.sqrt(n8 + n4 + 2)).half()
        st = codec.allocate_state(B, H, P, 128, 'cuda', layout=args.layout)
        call = lambda: codec.scan(x, dt, A, Bm, Cm, D, db, st, perm, basis, ls, pred, layout=args.layout)
        unit, work = 'us/token', float(L)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.steps):
        ev[0].record(s)
        call()
        ev[1].record(s)
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]) / 1e3)
    t = statistics.median(ts)
    val = work / t / 1e12 if unit == 'TFLOP/s' else (work / t / 1e9 if unit == 'GB/s' else t * 1e6 / work)
    extra = {}
    if args.case in ('sq3p25', 'ste'):
        B, L, H, P, G, K = STE_GEOMETRY
        extra = dict(geometry=dict(batch=B, tokens=L, heads=H, dim=P, groups=G, chunk=K),
                     cpu_baseline=ste_cpu_sample(args.case, B * H * P))
    print(json.dumps(dict(case=args.case, layout=args.layout if args.case == 'scan' else None, seconds=t,
                          value=val, unit=unit, steps=args.steps, rows=args.rows if args.case == 'gemv' else None,
                          layers=args.layers if args.case == 'decode' else None, **extra)), flush=True)


STE_GEOMETRY = (4, 512, 128, 64, 8, 32)   # batch, tokens, heads, dim, groups, chunk (training defaults)


def ste_cpu_sample(case, rows_full, tokens=64, heads=16, dim=64, chunk=32):
    """The CPU oracle (oracle/ste.py, one thread) on a bounded sample of the --case sq3p25 /
    ste workload: one sequence of `tokens` tokens over `heads` heads of one group; returns
    microseconds per token extrapolated to `rows_full` state rows."""
    from oracle import ste as ost
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, tokens, heads, dim)).astype(np.float16)
    dt = (rng.standard_normal((1, tokens, heads)) * 0.5).astype(np.float16)
    A = -(rng.random(heads) * 3 + 0.1).astype(np.float32)
    Bm = rng.standard_normal((1, tokens, 1, 128)).astype(np.float16)
    Cm = rng.standard_normal((1, tokens, 1, 128)).astype(np.float16)
    D = rng.standard_normal(heads).astype(np.float16)
    db = (rng.random(heads) * 3 - 4).astype(np.float16)
    perm = rng.permutation(128).astype(np.uint8)[None]
    t0 = time.perf_counter()
    if case == 'sq3p25':
        st = {k: np.zeros((1, heads, dim, n), np.uint8) for k, n in (('lo', 8), ('hi', 8), ('q4', 32))}
        st.update({k: np.zeros((1, heads, dim), np.float16) for k in ('s8', 's4')})
        ost.sq3p25_scan(x, dt, A, Bm, Cm, D, db, st, perm)
    else:
        ost.ste_backward(x, dt, A, Bm, Cm, D, db, perm, rng.standard_normal(x.shape).astype(np.float16), chunk)
    sec = time.perf_counter() - t0
    rows = heads * dim
    return dict(value=sec / tokens * rows_full / rows * 1e6, unit='us/token', cores=1, kind='port',
                sample=f'{tokens} tokens x {heads} heads x {dim} rows, extrapolated by rows', seconds=sec)


L2_FLUSH_BYTES = 256 << 20      # > 126 MB of L2


class L2Flush:
    """Writes a buffer larger than L2 before each timed launch of a small-operand kernel."""

    def __init__(self, device):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.zero_()


def timed(call, reps, flush=None, stream=None):
    """Median CUDA-event seconds of `call` on the current stream, L2 flushed before each.

    The flush (and a ~100 us device-side sleep behind it) is still running when the start
    event and the launch are enqueued, so host launch overhead never falls inside the
    measured interval."""
    s = stream or torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize()
        if flush:
            flush()
        torch.cuda._sleep(200000)
        e0.record(s)
        call()
        e1.record(s)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / 1e3)
    return statistics.median(ts)


@torch.no_grad()
def measure_config2(device, pk, reps=7):
    """FP4-G16 projections of one layer (in_proj 4096->18560, out_proj
    8192->4096) at M = 1, 8, 64, 256 through sq_fp4_linear (the reference's decoded-weight
    numerics), weights from seed 2; L2 flushed before every timed launch.  Algorithmic bytes
    = packed weights (0.5625 B/weight + 4) + X + Y; FLOPs = 2 M N K."""
    from sq325 import fp4 as F
    gen = torch.Generator(device=device).manual_seed(2)
    flush = L2Flush(device)
    rows = []
    for name, (N, K) in (('in_proj', (18560, 4096)), ('out_proj', (4096, 8192))):
        w = F.synthetic(N, K, gen, device)
        for M in (1, 8, 64, 256):
            x = torch.randn(M, K, device=device, generator=gen).half()
            call = lambda: F.linear(w, x)
            for _ in range(3):
                call()
            t = timed(call, reps, flush)
            byts = N * K * 9 // 16 + 4 + M * K * 2 + M * N * 2
            flop = 2.0 * M * N * K
            rows.append(dict(proj=name, M=M, us=t * 1e6, gbs=byts / t / 1e9, hbm_frac=byts / t / 1e9 / pk['hbm'],
                             tflops=flop / t / 1e12, tensor_frac=flop / t / 1e12 / pk['tf'],
                             path='skinny TMA GEMV (exact fp16 weights)' if M == 1 else
                             'tcgen05 FP4 linear (exact decode fused, weights as the A operand)'))
        del w
    return rows


@torch.no_grad()
def measure_config3(device, pk, steps=512, batch=64):
    """one Mamba-2 mixer layer (layout 32_32_64, no adapter, seed 3) decoding
    512 one-token steps at batch 64 from a zero SQ3.25 carry, fp16 N(0,1) inputs, the carry
    requantised every token.  The 512 steps are captured as one CUDA graph (each step: skinny
    in_proj, fused conv-step + scan, gated norm, skinny out_proj) and replayed; CUDA events.
    Bytes per step = both projections' packed weights + state rows read and written
    (52 B x 2) + conv ring read and written + the step's input and output rows."""
    from sq325 import model as M
    from sq325.state import PredictorState
    model = M.synthetic_model(seed=3, n_layer=1, vocab=256, device=device)
    ex = PredictorState(model, *M.synthetic_statics(('32_32_64',), seed=3, device=device)).install()
    try:
        ex.reset(batch)
        ex.reserve(batch)
        gen = torch.Generator(device=device).manual_seed(3)
        u = torch.randn(steps + 1, batch, 1, 4096, device=device, generator=gen).half()
        out = torch.empty(batch, 1, 4096, device=device, dtype=torch.float16)
        ex.mixer_forward(0, u[0], out)                      # position 0: prefill path, then one-token steps
        torch.cuda.synchronize()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for i in range(steps):
                    ex.mixer_forward(0, u[1 + i], out)
        torch.cuda.current_stream(device).wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        t = timed(g.replay, 3)
        ex.check()
        w = 18560 * 4096 * 9 // 16 + 4 + 4096 * 8192 * 9 // 16 + 4
        byts = w + batch * 8192 * 52 * 2 + batch * 4 * 10240 * 2 * 2 + batch * 4096 * 2 * 2
        finite = bool(torch.isfinite(out).all())
        del g
    finally:
        ex.close()
    return dict(steps=steps, batch=batch, us_per_step=t / steps * 1e6, tokens_per_s=steps * batch / t,
                bytes_per_step=byts, gbs=byts * steps / t / 1e9, hbm_frac=byts * steps / t / 1e9 / pk['hbm'],
                output_finite=finite, launches_per_step=4)


@torch.no_grad()
def measure_config5(ex, wins_rng_seed, device, pk, prompt_len=1024, new_tokens=256):
    """greedy generation on the config-4 model (Resurface on): a 1024-token
    Zipf prompt, then 256 new tokens, at batch 1 (persistent decode kernel, one launch for
    all tokens; also the multi-kernel step as CUDA-graph replays, in both projection
    numerics) and batch 32 (CUDA-graph replays).  Prefill rates count prompt tokens."""
    rng = np.random.default_rng(wins_rng_seed)
    prompts = torch.from_numpy(zipf_tokens(32 * prompt_len, rng).reshape(32, prompt_len)).to(device)
    res = {}
    roof1 = pk['hbm'] * 1e9 / DECODE_BYTES_B1
    for batch in (1, 32):
        p = prompts[:batch].contiguous()
        ex.backbone(p, reset=True)                                  # warm-up
        t_pre = timed(lambda: ex.backbone(p, reset=True), 2)
        h = ex.backbone(p, reset=True)[:, -1]
        tok = ex.greedy(h).clone()
        n = new_tokens - 1
        bytes_step = DECODE_FIXED_BYTES + batch * DECODE_PER_SEQ_BYTES
        r = dict(prefill_tokens_per_s=batch * prompt_len / t_pre,
                 prefill_tflops=FLOP_PER_TOKEN_BACKBONE * batch * prompt_len / t_pre / 1e12,
                 bytes_per_step=bytes_step, roofline_tokens_per_s=batch * pk['hbm'] * 1e9 / bytes_step)
        if batch == 1:
            ex.decode_persistent(tok, n)                            # warm-up at full length
            t = timed(lambda: ex.decode_persistent(tok, n), 1)
            ex.check()
            r.update(tokens_per_s=n / t, ms_per_token=t / n * 1e3, frac=(n / t) / roof1, kernel='persistent')
            ex.capture_decode(tok)
            ex.replay_decode(n)
            tg = timed(lambda: ex.replay_decode(n), 1)
            r['graph_replay_tokens_per_s'] = n / tg
            ex.set_exact_projections(True)
            try:
                ex.capture_decode(tok)
                ex.replay_decode(8)
                te = timed(lambda: ex.replay_decode(n), 1)
                ex.decode_persistent(tok, n)
                tpe = timed(lambda: ex.decode_persistent(tok, n), 1)
                ex.check()
            finally:
                ex.set_exact_projections(False)
            r['exact_graph_replay_tokens_per_s'] = n / te
            r['exact_tokens_per_s'] = n / tpe
        else:
            ex.capture_decode(tok)
            ex.replay_decode(8)
            t = timed(lambda: ex.replay_decode(n), 1)
            ex.check()
            r.update(tokens_per_s=batch * n / t, ms_per_step=t / n * 1e3,
                     frac=(batch * n / t) / r['roofline_tokens_per_s'], kernel='graph replay')
        res[f'batch{batch}'] = r
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=4)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='native', choices=['native', 'reference'])
    ap.add_argument('--ref-tokens', type=int, default=2048)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-extras', action='store_true',
                    help='skip the config 2 / 3 / 5 measurements of the one-GPU line')
    ap.add_argument('--rows', type=int, default=1, help='M of --case gemv')
    ap.add_argument('--case', choices=['gemm', 'scan', 'decode', 'gemv', 's16', 'sq3p25', 'ste'], default=None,
                    help='time one kernel on a small case (for ncu captures) instead of the bench')
    ap.add_argument('--layout', default='32_32_64', help='scan layout of --case scan')
    ap.add_argument('--layers', type=int, default=4, help='layers of --case decode')
    ap.add_argument('--vocab', type=int, default=32768, help='vocabulary of --case decode')
    args = ap.parse_args()
    if args.case:
        if args.case == 'scan' and args.layout == 'all':
            from sq325.codec import LAYOUTS
            for layout in LAYOUTS:
                args.layout = layout
                run_case(args)
        else:
            run_case(args)
        return
    args.steps_ref = min(args.steps, 3)
    args.warmup_ref = 1 if args.warmup > 0 else 0
    if args.impl == 'reference':
        rank = int(os.environ.get('RANK', 0))
        run_reference(args, rank, int(os.environ.get('WORLD_SIZE', 1)))
        return
    rank, world, local = dist_init(args.gpus)
    device = torch.device('cuda', local)
    import torch.distributed as dist
    from sq325 import scoring

    model, ex, wins, setup_s = build_workload(rank, device)
    B, T = WINDOWS_PER_GPU, SEQLEN
    ex.reserve(B * T)
    ids_dev = torch.from_numpy(wins).to(device)
    # The global window list: rank r owns windows r, r + N, r + 2N, ... (the round-robin split
    # of evaluate_ppl); each rank fills in its own 16 windows, on the device for `value` and
    # in pinned host memory for `e2e`.  Other ranks' entries are never touched.
    starts = [(i * world + rank) * (SEQLEN + 1) for i in range(B)]
    dev_windows = [(0, None)] * (world * B)
    host_windows = [(0, None)] * (world * B)
    for i in range(B):
        dev_windows[i * world + rank] = (starts[i], ids_dev[i])
        host_windows[i * world + rank] = (starts[i], torch.from_numpy(wins[i]).pin_memory())

    def step(windows):
        # the public scoring API: local windows batched, one NLL all-reduce (+ the per-window
        # records gathered on the host) across ranks
        return scoring.evaluate_ppl(ex, windows, batch_windows=B, rank=rank, world=world)

    for _ in range(args.warmup):
        step(dev_windows)
    torch.cuda.synchronize()
    ex.check()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ex.time_projection_gemm(True)        # CUDA events around each in_proj GEMM launch of the timed steps
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(s)
    for _ in range(args.steps):
        res = step(dev_windows)
    e1.record(s)
    torch.cuda.synchronize()
    gemm_in_step_s, gemm_in_step_n = ex.projection_gemm_time()
    ex.time_projection_gemm(False)
    if world > 1:
        dist.barrier()
    elapsed = e0.elapsed_time(e1) / 1e3
    clk = clocks.stop()
    ex.check()
    t = torch.tensor([elapsed], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = float(t)
    tokens_all = world * B * T * args.steps
    value = tokens_all / elapsed
    assert res['target_tokens'] == world * B * T and len(res['windows']) == world * B and math.isfinite(res['ppl'])

    # e2e: the same API from pinned host windows (H2D of the windows and D2H of the NLL sums
    # inside the timed region, every step)
    h2d = B * (SEQLEN + 1) * 8
    d2h = B * 8
    step(host_windows)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_steps = max(1, min(args.steps, 2))
    for _ in range(e2e_steps):
        step(host_windows)
    torch.cuda.synchronize()
    e2e_el = time.perf_counter() - t0
    te = torch.tensor([e2e_el], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * B * T * e2e_steps / float(te)

    # dominant kernel roofline: the in_proj GEMM launches of the timed steps (CUDA events on
    # the launching stream inside the timed region), against the sustained peak since they run
    # inside a seconds-long power-capped step; the same GEMM timed alone (burst) for context
    pk = peaks()
    gemm_flop = 2.0 * B * T * 18560 * 4096
    gemm_alone_s, _ = time_gemm_kernel(model, B * T, device)
    in_step = gemm_in_step_n == N_LAYER * args.steps   # one M = B*T launch per layer and step
    gemm_s = gemm_in_step_s / gemm_in_step_n if in_step else gemm_alone_s
    achieved = gemm_flop / gemm_s / 1e12
    gemm_peak = pk['tf_sus'] if in_step else pk['tf']

    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        extras['config5_generation'] = measure_config5(ex, 5, device, pk)
        extras['config2_fp4_linear'] = measure_config2(device, pk)
        extras['config3_layer_step'] = measure_config3(device, pk)
    decode = None
    if 'config5_generation' in extras:
        b1 = extras['config5_generation']['batch1']
        decode = dict(tokens_per_s=b1['tokens_per_s'], ms_per_token=b1['ms_per_token'],
                      roofline_tokens_per_s=b1['roofline_tokens_per_s'], frac=b1['frac'],
                      bytes_per_token=DECODE_BYTES_B1, graph_replay_tokens_per_s=b1['graph_replay_tokens_per_s'],
                      exact_graph_replay_tokens_per_s=b1['exact_graph_replay_tokens_per_s'],
                      exact_tokens_per_s=b1['exact_tokens_per_s'],
                      exact_frac=b1['exact_tokens_per_s'] / b1['roofline_tokens_per_s'],
                      note='config 5: 1024-token prompt, 255 greedy tokens in one persistent cooperative launch '
                           '(factored-scale projections, the default for decode steps; exact_* = the same '
                           'launch with the exact per-weight fp16 decode, the reference numerics); graph '
                           'replays = the multi-kernel step as CUDA graphs, in both numerics')

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        per_tok, info = cpu_sample(tokens=args.ref_tokens)
        cpu = dict(value=1.0 / per_tok, unit=UNIT, cores=os.cpu_count(), kind='port',
                   sample=f"oracle port, 1 window x {info['tokens']} tokens through {info['layers']} layers + "
                          f"lm_head/CE over a {info['vocab_slice']}-row vocab slice, extrapolated to 56 layers and "
                          f"256000 rows; {info['seconds']:.1f} s of CPU work")
    if rank == 0:
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=elapsed / args.steps * 1e3, higher_is_better=True, scaling='weak', vs_baseline=None,
            dtype='fp16 (fp32 accumulate)', data='synthetic',
            config=workload_config(world, B, T),
            e2e=dict(value=e2e_value, unit=UNIT, h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h),
            roofline=dict(bound='tensor', kernel='tcgen05 in_proj GEMM (M=%d,N=18560,K=4096)' % (B * T),
                          achieved=achieved, peak=gemm_peak, unit='TFLOP/s', frac=achieved / gemm_peak,
                          traffic=GEMM_TRAFFIC_BYTES,
                          peak_source=pk['src'] + (' bf16_tflops_sustained (launches timed inside the step)' if in_step
                                                   else ' bf16_tflops (burst; launch count differed, timed alone)'),
                          launches_timed=gemm_in_step_n, ms_per_launch=gemm_s * 1e3,
                          alone=dict(ms=gemm_alone_s * 1e3, achieved=gemm_flop / gemm_alone_s / 1e12, peak=pk['tf'],
                                     frac=gemm_flop / gemm_alone_s / 1e12 / pk['tf'],
                                     note='same GEMM timed alone after the step, burst peak')),
            step_roofline=dict(flop_per_token=FLOP_PER_TOKEN,
                               achieved_tflops=FLOP_PER_TOKEN * value / world / 1e12,
                               frac=FLOP_PER_TOKEN * value / world / 1e12 / pk['tf_sus']),
            decode_b1=decode, cpu_baseline=cpu, clocks=clk,
            gpu_launches=launches_per_step(B * T) * args.steps,
            setup_seconds=setup_s, **extras)
        print(json.dumps(line), flush=True)
    ex.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
