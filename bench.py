"""Benchmark of the cuda_kda hot path: chunkwise KDA forward + VJP, B8 H12 T1568 d64 bf16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one kda_fwd (saving the per-chunk states) + one kda_bwd over one batch of seeded
synthetic inputs with BASELINE config 2's shapes and distributions (q, k L2-normalised
N(0,1); v N(0,1); beta sigmoid(N(0,1)); g -softplus(N(0,1)) float32; S0 N(0, 0.1^2);
dO N(0,1) bf16; dS_T N(0,1)).  Scaling is strong: the fixed B8 x H12 problem's 96 (b, h)
sequences are split over the N ranks (96/N each, contiguous over b then h); nothing crosses
GPUs inside the op.  ``value`` = 12,544 tokens (B*T) per step / max-over-ranks device time.
The same line carries a weak-scaling leg (every rank its own B8 x H12), config 1 (inference
forward), config 4 (streaming D = 128, heads over ranks) and config 3 (the full model's DP
training step) as nested keys.

``--impl reference`` times the CPU restatement of the reference's ``compiled`` path
(the oracle port: MLX cannot run here) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, H, T, D, CHUNK = 8, 12, 1568, 64, 64
METRIC = "KDA fwd+bwd tokens/sec/GPU (B8 H12 T1568 d64 bf16) and % of roofline"
UNIT = "tokens/s"
E2E_WINDOWS = 5  # timed windows of K steps for the end-to-end leg (median reported)
# algorithmic (compulsory) HBM bytes per call over the whole B8 H12 problem: every input read
# once and every output written once (forward: q, k, v, o bf16, g fp32, beta bf16, S0 and S_T
# fp32; backward: q, k, v, g, beta, S0, dO, dS_T read, dq, dk, dv, dg, dbeta, dS0 written)
FWD_BYTES = 119_052_288
BWD_BYTES = 217_264_128
FLOPS_FWD_PER_TOKHEAD = 40_960
FLOPS_FWDBWD_PER_TOKHEAD = 139_264


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------------------
# CPU reference arm (oracle port of the reference's `compiled` path + its step backward)
# ---------------------------------------------------------------------------------------
def _cpu_pair(args):
    seed, pair = args
    import numpy as np
    from mlx_vit_b200.synthetic import make_inputs
    from oracle import kda_oracle as O
    inp = make_inputs(1, T, 1, D, seed=seed * 1000 + pair, state_std=0.1)
    for k in ("q", "k", "v", "beta", "do"):  # bf16-rounded operands, as the GPU sees them
        a = inp[k].astype(np.float32)
        inp[k] = (a.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    O.compiled_forward(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["state"])
    O.step_backward(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["state"],
                    inp["do"], inp["dst"])
    return pair


def cpu_reference(steps: int, warmup: int):
    """Times the oracle on (b, h) sequences of the config, one sequence per worker process
    (single-threaded BLAS each), all host cores.  Returns (tokens/s, cores, sample, secs)."""
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    workers = max(1, min(cores, B * H))
    pairs = B * H if workers >= 16 else min(B * H, 2 * workers)
    env_keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    old = {k: os.environ.get(k) for k in env_keys}
    for k in env_keys:
        os.environ[k] = "1"
    try:
        ctx = mp.get_context("spawn")
        with ctx.Pool(workers) as pool:
            for i in range(warmup):
                pool.map(_cpu_pair, [(i, p) for p in range(min(pairs, workers))])
            times = []
            for s in range(steps):
                t0 = time.perf_counter()
                pool.map(_cpu_pair, [(100 + s, p) for p in range(pairs)])
                times.append(time.perf_counter() - t0)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    tok = pairs * T / H  # tokens (each token covers H heads)
    tsec = statistics.median(times)
    sample = (f"{pairs} of the {B * H} (b,h) sequences of B8 H12 T1568 d64 (bf16-rounded "
              f"inputs, fp32 numpy), fwd (compiled-path restatement) + step-backward VJP, "
              f"{workers} worker processes x 1 BLAS thread, median of {steps}")
    return tok / tsec, workers, sample, tsec


# ---------------------------------------------------------------------------------------
# clocks sampler
# ---------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        # nvidia-smi numbers GPUs in PCI order regardless of CUDA_VISIBLE_DEVICES; its UUID
        # names the GPU this process runs on unambiguously
        import torch
        self.idx = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.proc or not self.f:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.f.flush()
        rows = []
        with open(self.f.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------
def fused_gates_leg(args, L, dev, inp, calls, flush):
    """The layer's gates + recurrence, fwd+bwd, two ways on this rank's share (gate init as the
    reference's: A = e^{A_log} uniform in [1, 16], f and b standard normal projections):
    fused (kda_fwd_gated / kda_bwd_gated) and unfused (torch evaluates g, beta and their VJP
    around kda_fwd / kda_bwd).  Both CUDA-graph replayed, L2 flushed before each step."""
    import ctypes
    import torch
    from mlx_vit_b200 import _lib
    from mlx_vit_b200.kda import _desc, _ptr, _gate_struct
    from mlx_vit_b200.shard import max_over_ranks
    q, k, v, S0, do, dst = (inp[n] for n in ("q", "k", "v", "state", "do", "dst"))
    Br, _, Hr, _ = q.shape
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    f = torch.randn(Br, T, Hr, D, generator=gen, device=dev).to(torch.bfloat16)
    bl = torch.randn(Br, T, Hr, generator=gen, device=dev).to(torch.bfloat16)
    A_log = torch.log(torch.rand(Hr, generator=gen, device=dev) * 15 + 1)
    dtb = torch.zeros(Hr * D, device=dev)
    gate = _gate_struct(f, A_log, dtb, bl, False)
    gdesc = _desc(q, bl, CHUNK, 0)
    df, dbl = torch.empty_like(f), torch.empty_like(bl)
    dA, ddtb = torch.empty(Hr, device=dev), torch.empty(Hr * D, device=dev)
    c = calls
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fused():
        _lib.check(L.kda_fwd_gated(ctypes.byref(gdesc), _ptr(q), _ptr(k), _ptr(v), ctypes.byref(gate),
                                   _ptr(S0), _ptr(c.o), _ptr(c.S_T), _ptr(c.saved), _ptr(c.wsf), c.nwsf,
                                   stream()), "kda_fwd_gated")
        _lib.check(L.kda_bwd_gated(ctypes.byref(gdesc), _ptr(q), _ptr(k), _ptr(v), ctypes.byref(gate),
                                   _ptr(S0), _ptr(c.saved), _ptr(do), _ptr(dst), _ptr(c.dq), _ptr(c.dk),
                                   _ptr(c.dv), _ptr(df), _ptr(dbl), _ptr(dA), _ptr(ddtb), _ptr(c.ds0),
                                   _ptr(c.ws), c.nws, stream()), "kda_bwd_gated")

    g = torch.empty(Br, T, Hr, D, device=dev)
    beta = torch.empty(Br, T, Hr, device=dev, dtype=torch.bfloat16)
    dg, dbeta = torch.empty_like(g), torch.empty_like(beta)
    pdesc = _desc(q, beta, CHUNK, 0)

    def unfused():
        x = f.float() + dtb.view(Hr, D)
        A = torch.exp(A_log).view(1, 1, Hr, 1)
        g.copy_(-A * torch.nn.functional.softplus(x))
        sb = torch.sigmoid(bl.float())
        beta.copy_(sb)
        _lib.check(L.kda_fwd(ctypes.byref(pdesc), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                             _ptr(S0), _ptr(c.o), _ptr(c.S_T), _ptr(c.saved), _ptr(c.wsf), c.nwsf, stream()),
                   "kda_fwd")
        _lib.check(L.kda_bwd(ctypes.byref(pdesc), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                             _ptr(S0), _ptr(c.saved), _ptr(do), _ptr(dst), _ptr(c.dq), _ptr(c.dk), _ptr(c.dv),
                             _ptr(dg), _ptr(dbeta), _ptr(c.ds0), _ptr(c.ws), c.nws, stream()), "kda_bwd")
        dfx = dg * (-A) * torch.sigmoid(x)
        df.copy_(dfx)
        dA.copy_((dg * g).sum(dim=(0, 1, 3)))
        ddtb.copy_(dfx.sum(dim=(0, 1)).view(-1))
        dbl.copy_(dbeta.float() * sb * (1 - sb))

    out = {}
    for name, fn in (("fused", fused), ("unfused", unfused)):
        (ms,) = graph_time([fn], args.steps, args.warmup, flush)
        out[name + "_ms_per_step"] = round(max_over_ranks(statistics.mean(ms), dev), 4)
    out["tokens_per_s"] = round(B * T / (out["fused_ms_per_step"] / 1e3), 1)
    out["workload"] = ("cfg2 shape (this rank's share), gates from bf16 f [B,T,H,D] and b [B,T,H], "
                       "A = e^{A_log} in [1, 16] (reference init), dt_bias 0; fwd+bwd incl. df, db, "
                       "dA_log, ddt_bias")
    return out


def streaming_d128_leg(args, L, dev, flush, rank, world):
    """cfg4 (streaming inference): B1 H16 D128 chunk 64, T = 16384 as 4 segments of 4096 with
    the state carried, the 16 heads sharded over the ranks (16/N each); forward only, each
    segment one kda_fwd call.  CUDA-graph replayed, L2 flushed per step, max over ranks."""
    import ctypes
    import torch
    from mlx_vit_b200 import _lib
    from mlx_vit_b200.kda import _desc, _ptr
    from mlx_vit_b200.shard import max_over_ranks, shard_range
    from mlx_vit_b200.synthetic import make_inputs_torch
    lo, hi = shard_range(16, world, rank)
    Bs, Hs, Ts, Ds, nseg = 1, max(1, hi - lo), 4096, 128, 4
    inp = make_inputs_torch(Bs, Ts * nseg, Hs, Ds, seed=77 + rank, device=dev, dtype=torch.bfloat16)
    seg = [{n: inp[n][:, Ts * i:Ts * (i + 1)].contiguous() for n in ("q", "k", "v", "g", "beta")}
           for i in range(nseg)]
    desc = _desc(seg[0]["q"], seg[0]["beta"], CHUNK, 0)
    nws = L.kda_workspace_bytes(ctypes.byref(desc), 0)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
    states = [inp["state"].clone()] + [torch.empty_like(inp["state"]) for _ in range(nseg)]
    outs = [torch.empty_like(x["q"]) for x in seg]
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def step():
        for i, x in enumerate(seg):
            _lib.check(L.kda_fwd(ctypes.byref(desc), _ptr(x["q"]), _ptr(x["k"]), _ptr(x["v"]), _ptr(x["g"]),
                                 _ptr(x["beta"]), _ptr(states[i]), _ptr(outs[i]), _ptr(states[i + 1]),
                                 None, _ptr(ws), nws, stream()), "kda_fwd")
    c0 = L.kda_launch_counter()
    step()
    launches = L.kda_launch_counter() - c0
    (ms,) = graph_time([step], args.steps, args.warmup, flush)
    t = max_over_ranks(statistics.mean(ms), dev)

    # decoding: one token per call with the state carried, the step kernel (kda_fwd_recurrent)
    # against the chunked forward (one padded chunk per call); 64 tokens per timed graph
    ndec = 64
    xd = {n: inp[n][:, :ndec].contiguous() for n in ("q", "k", "v", "g", "beta")}
    tok = [{n: xd[n][:, i:i + 1] for n in xd} for i in range(ndec)]
    sd = [inp["state"].clone()] + [torch.empty_like(inp["state"]) for _ in range(ndec)]
    od = [torch.empty_like(x["q"]) for x in tok]
    d1 = _desc(tok[0]["q"], tok[0]["beta"], CHUNK, 0)
    nws1 = L.kda_workspace_bytes(ctypes.byref(d1), 0)
    ws1 = torch.empty(max(nws1, 16), dtype=torch.uint8, device=dev)

    def decode(recurrent):
        for i, x in enumerate(tok):
            a = (ctypes.byref(d1), _ptr(x["q"]), _ptr(x["k"]), _ptr(x["v"]), _ptr(x["g"]), _ptr(x["beta"]),
                 _ptr(sd[i]), _ptr(od[i]), _ptr(sd[i + 1]))
            if recurrent:
                _lib.check(L.kda_fwd_recurrent(*a, stream()), "kda_fwd_recurrent")
            else:
                _lib.check(L.kda_fwd(*a, None, _ptr(ws1), nws1, stream()), "kda_fwd")
    dec = {}
    for name, rec in (("recurrent", True), ("chunked", False)):
        (dms,) = graph_time([lambda: decode(rec)], max(1, args.steps // 4), 2, flush)
        dec[name + "_us_per_token"] = round(max_over_ranks(statistics.mean(dms), dev) * 1e3 / ndec, 2)
    return {"decode_d128": dict(dec, workload=f"one token per call, B1 H{Hs} D128, state carried "
                                              "(CUDA graph of 64 calls)"),
            "workload": f"cfg4: B1 H16 D128 chunk64, 4 x 4096 tokens with the state carried (bf16 "
                        f"I/O, fp32 g/state), forward; {Hs} heads per GPU over {world} GPU(s)",
            "ms_per_step": round(t, 4), "tokens_per_s": round(Bs * Ts * nseg / (t / 1e3), 1),
            "gpu_launches_per_step": int(launches)}


def rank_shape(world, rank):
    """This rank's share of the B8 x H12 problem as a (B_r, H_r) batch: B/N batch rows of all
    heads when N divides B (pairs contiguous over b then h), else a run of the 96 (b, h) pairs
    laid out as the heads of one row (the pairs are independent, so the layout is immaterial)."""
    from mlx_vit_b200.shard import shard_range
    if B % world == 0:
        return B // world, H
    lo, hi = shard_range(B * H, world, rank)
    return 1, hi - lo


def graph_time(fns, steps, warmup, flush, events_per_fn=False):
    """Captures each callable in ``fns`` in its own CUDA graph and replays them back to back per
    step, L2 flushed before each step; returns per-callable lists of CUDA-event milliseconds."""
    import torch
    for _ in range(max(3, warmup)):
        for f in fns:
            f()
    torch.cuda.synchronize()
    graphs = []
    for f in fns:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            f()
        graphs.append(gr)
    for _ in range(max(3, warmup)):
        for gr in graphs:
            gr.replay()
    torch.cuda.synchronize()
    ms = [[] for _ in fns]
    for _ in range(steps):
        flush.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(fns) + 1)]
        ev[0].record()
        for i, gr in enumerate(graphs):
            gr.replay()
            ev[i + 1].record()
        ev[-1].synchronize()
        for i in range(len(fns)):
            ms[i].append(ev[i].elapsed_time(ev[i + 1]))
    return ms


class KdaCalls:
    """Preallocated kda_fwd / kda_bwd calls over one (B_r, T, H_r) batch on the current stream."""

    def __init__(self, L, inp, dev):
        import ctypes
        import torch
        from mlx_vit_b200.kda import _desc, _ptr
        self.L, self.inp, self._ptr, self.ct = L, inp, _ptr, ctypes
        q, beta, g, S0 = inp["q"], inp["beta"], inp["g"], inp["state"]
        Br, _, Hr, _ = q.shape
        self.desc = _desc(q, beta, CHUNK, 0)
        by = ctypes.byref(self.desc)
        self.o = torch.empty_like(q)
        self.S_T = torch.empty((Br, Hr, D, D), dtype=torch.float32, device=dev)
        self.saved = torch.empty(L.kda_saved_bytes(by), dtype=torch.uint8, device=dev)
        self.nws = L.kda_workspace_bytes(by, 1)
        self.ws = torch.empty(max(self.nws, 16), dtype=torch.uint8, device=dev)
        self.nwsf = L.kda_workspace_bytes(by, 0)
        self.wsf = torch.empty(max(self.nwsf, 16), dtype=torch.uint8, device=dev)
        self.dq, self.dk, self.dv = (torch.empty_like(q) for _ in range(3))
        self.dg, self.db, self.ds0 = torch.empty_like(g), torch.empty_like(beta), torch.empty_like(S0)

    def _stream(self):
        import torch
        return self.ct.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fwd(self, save=True):
        from mlx_vit_b200 import _lib
        P, x = self._ptr, self.inp
        st = self.L.kda_fwd(self.ct.byref(self.desc), P(x["q"]), P(x["k"]), P(x["v"]), P(x["g"]),
                            P(x["beta"]), P(x["state"]), P(self.o), P(self.S_T),
                            P(self.saved) if save else None, P(self.wsf), self.nwsf, self._stream())
        _lib.check(st, "kda_fwd")

    def bwd(self):
        from mlx_vit_b200 import _lib
        P, x = self._ptr, self.inp
        st = self.L.kda_bwd(self.ct.byref(self.desc), P(x["q"]), P(x["k"]), P(x["v"]), P(x["g"]),
                            P(x["beta"]), P(x["state"]), P(self.saved), P(x["do"]), P(x["dst"]),
                            P(self.dq), P(self.dk), P(self.dv), P(self.dg), P(self.db), P(self.ds0),
                            P(self.ws), self.nws, self._stream())
        _lib.check(st, "kda_bwd")


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from mlx_vit_b200 import _lib, cuda_kda
    from mlx_vit_b200.shard import max_over_ranks
    from mlx_vit_b200.synthetic import make_inputs_torch

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    dt = torch.bfloat16
    Br, Hr = rank_shape(world, rank)
    pairs_r = Br * Hr
    inp = make_inputs_torch(Br, T, Hr, D, seed=1234 + rank, device=dev, dtype=dt, state_std=0.1)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2
    calls = KdaCalls(L, inp, dev)

    # ---- e2e through the public API with host buffers (pinned), copies inside timing; first,
    #      before any CUDA graph or other leg of this process ----
    # Every step copies this rank's inputs host->device, runs cuda_kda forward + autograd
    # backward and copies all outputs and gradients device->host.  Consecutive steps overlap the
    # way a data pipeline does: step i + 2's inputs go up (copy stream) and step i's results come
    # down (second copy stream) while step i + 1 computes; PCIe carries both directions at once.
    host = {n: x.cpu().pin_memory() for n, x in inp.items()}
    h2d = sum(x.numel() * x.element_size() for x in host.values())
    LEAVES = ("q", "k", "v", "g", "beta", "state")
    main = torch.cuda.current_stream(dev)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dev_in = [{n: torch.empty(x.shape, dtype=x.dtype, device=dev) for n, x in host.items()} for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    outs_host = [None, None]
    d2h = 0

    def upload(i, after=None):
        buf = i & 1
        with torch.cuda.stream(s_up):
            if after is not None:
                s_up.wait_event(after)
            s_up.wait_event(in_free[buf])
            for n, x in host.items():
                dev_in[buf][n].copy_(x, non_blocking=True)
            in_ready[buf].record(s_up)

    def compute_download(i):
        nonlocal d2h
        buf = i & 1
        main.wait_event(in_ready[buf])
        d = dev_in[buf]
        leaves = {n: d[n].detach().requires_grad_(True) for n in LEAVES}
        o, S_T = cuda_kda(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"],
                          leaves["state"], chunk_size=CHUNK)
        torch.autograd.backward([o, S_T], [d["do"], d["dst"]])
        res = [o.detach(), S_T.detach()] + [leaves[n].grad for n in LEAVES]
        in_free[buf].record(main)
        if outs_host[buf] is None:
            outs_host[buf] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
        with torch.cuda.stream(s_down):
            s_down.wait_event(in_free[buf])
            for hdst, r in zip(outs_host[buf], res):
                r.record_stream(s_down)
                hdst.copy_(r, non_blocking=True)
        d2h = sum(r.numel() * r.element_size() for r in res)

    def pipeline(n, start=None):
        for e in in_free:
            e.record(main)
        upload(0, start)
        if n > 1:
            upload(1, start)
        for i in range(n):
            compute_download(i)
            if i + 2 < n:
                upload(i + 2)
        main.wait_stream(s_down)

    pipeline(max(3, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # Host-driven copies see the host's other load (PCIe, memory, CPU): the same code measured
    # 1.0-4.5 M tokens/s between single windows on one box.  So E2E_WINDOWS consecutive windows
    # of K steps each are timed (device events, max over ranks) and the median is reported, with
    # every window listed beside it.
    e2e_windows = []
    for _ in range(E2E_WINDOWS):
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(main)
        pipeline(args.steps, start=e0)
        e1.record(main)
        torch.cuda.synchronize()
        e2e_windows.append(B * T * args.steps / (max_over_ranks(e0.elapsed_time(e1), dev) / 1e3))
    e2e_value = sorted(e2e_windows)[len(e2e_windows) // 2]
    del dev_in, outs_host, host


    # ---- headline: fwd (saving the record) + bwd on this rank's share, CUDA graphs ----
    c0 = L.kda_launch_counter()
    calls.fwd()
    calls.bwd()
    launches_per_step = L.kda_launch_counter() - c0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(dev) as clk:
        fwd_ms, bwd_ms = graph_time([calls.fwd, calls.bwd], args.steps, args.warmup, flush)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = launches_per_step * args.steps
    total_ms = max_over_ranks(sum(fwd_ms) + sum(bwd_ms), dev)
    ms_per_step = total_ms / args.steps
    tokens_step = B * T  # the whole problem, over all ranks
    value = tokens_step * args.steps / (total_ms / 1e3)
    fwd_avg = max_over_ranks(statistics.mean(fwd_ms), dev)
    bwd_avg = max_over_ranks(statistics.mean(bwd_ms), dev)

    # ---- config 1: inference forward (no saved record) on the same share ----
    (inf_ms,) = graph_time([lambda: calls.fwd(save=False)], args.steps, args.warmup, flush)
    inf_avg = max_over_ranks(statistics.mean(inf_ms), dev)

    # ---- weak scaling (N > 1): every rank its own full B8 x H12 ----
    weak = None
    if world > 1:
        winp = make_inputs_torch(B, T, H, D, seed=4321 + rank, device=dev, dtype=dt, state_std=0.1)
        wc = KdaCalls(L, winp, dev)
        wf, wb = graph_time([wc.fwd, wc.bwd], args.steps, args.warmup, flush)
        wms = max_over_ranks((sum(wf) + sum(wb)) / args.steps, dev)
        weak = {"value": round(B * T * world / (wms / 1e3), 1), "unit": UNIT, "ms_per_step": round(wms, 4),
                "workload": "every rank its own B8 H12 T1568 (global batch 8 N)"}
        del wc, winp


    fused = fused_gates_leg(args, L, dev, inp, calls, flush)
    streaming = streaming_d128_leg(args, L, dev, flush, rank, world)

    cfg3 = None
    if not args.skip_cfg3:
        torch.cuda.empty_cache()
        cfg3 = run_cfg3(args, rank, world, local_rank, steps=min(args.steps, 5))

    if rank != 0:
        return None
    hbm, tfl, src = peaks()
    share = pairs_r / (B * H)  # the rank's share of the algorithmic bytes (rank 0's)
    # dominant call: the longer of the two (the backward is two launches)
    if bwd_avg >= fwd_avg:
        dom, dom_ms, dom_bytes = "kda_bwd", bwd_avg, BWD_BYTES * share
    else:
        dom, dom_ms, dom_bytes = "kda_fwd", fwd_avg, FWD_BYTES * share
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    whole = (FWD_BYTES + BWD_BYTES) * share / (ms_per_step / 1e3) / 1e9
    inf_gbs = FWD_BYTES * share / (inf_avg / 1e3) / 1e9
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config-2 distributions)",
        "config": {"workload": "cfg2: chunkwise KDA fwd+VJP, B8 H12 T1568 dk=dv=64 chunk64, bf16 "
                               "I/O, fp32 g/state; the 96 (b,h) sequences split over the GPUs",
                   "global_batch": B, "H": H, "T": T, "D": D, "chunk": CHUNK,
                   "per_rank_shape": [Br, T, Hr, D], "parallelism": f"bxh-shard x{world} (strong)",
                   "l2": "flushed (256 MB write) before every timed step"},
        "per_gpu_tokens_per_s": round(value / world, 1),
        "fwd_ms": round(fwd_avg, 4), "bwd_ms": round(bwd_avg, 4),
        "hbm_frac_whole_step": round(whole / hbm, 4),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "algorithmic_bytes_per_launch": int(dom_bytes), "traffic": None},
        "gpu_launches": int(launches),
        "cfg1_inference_fwd": {"ms": round(inf_avg, 4),
                               "tokens_per_s": round(tokens_step / (inf_avg / 1e3), 1),
                               "hbm_gbs": round(inf_gbs, 1), "hbm_frac": round(inf_gbs / hbm, 4),
                               "algorithmic_bytes": int(FWD_BYTES * share),
                               "workload": "cfg1: kda_fwd without the saved record, S0 given, same shard"},
        "weak_scaling": weak,
        "fused_gates": fused,
        "streaming_d128": streaming,
        "cfg3": cfg3,
        "clocks": clocks,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "windows": [round(x, 1) for x in e2e_windows],
                "d2h_bytes_per_step": int(d2h),
                "path": "mlx_vit_b200.cuda_kda autograd fwd+bwd from pinned host buffers, all "
                        "outputs and gradients copied back; consecutive "
                        "steps' copies overlap compute (upload, compute, download on three "
                        "streams); per-rank bytes; value = median of the timed windows "
                        "of K steps each"},
    }
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf) and world == 1:
        try:
            with open(tf) as f:
                tr = json.load(f).get(dom)
            if tr:
                line["roofline"]["traffic"] = tr
                line["roofline"]["traffic_note"] = "ncu dram__bytes_read.sum + write.sum of the call's kernels"
        except Exception:
            pass
    if world == 1 and not args.no_cpu_baseline:
        v, cores, sample, _ = cpu_reference(steps=5, warmup=1)
        line["cpu_baseline"] = {"value": round(v, 1), "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": sample}
    return line


def kernel_only(args):
    """Launches only the library calls on the benchmark workload (a driver for ncu)."""
    import torch
    from mlx_vit_b200 import kda_forward, kda_backward
    from mlx_vit_b200.synthetic import make_inputs_torch
    dev = torch.device("cuda", 0)
    if args.kernel_only == "stream":  # the D = 128 streaming forward: cfg4's share of one GPU
        x = make_inputs_torch(1, 4096, 2, 128, seed=77, device=dev, dtype=torch.bfloat16)
        st = x["state"]
        for _ in range(args.warmup + args.steps):
            for _ in range(4):
                _, st, _ = kda_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], st, CHUNK)
        torch.cuda.synchronize()
        return 0
    if args.kernel_only == "recurrent":  # token-by-token decode: cfg4's heads, 64 tokens per call
        x = make_inputs_torch(1, 64, 16, 128, seed=77, device=dev, dtype=torch.bfloat16)
        from mlx_vit_b200 import kda_recurrent
        st = x["state"]
        for _ in range(args.warmup + args.steps):
            _, st = kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], st)
        torch.cuda.synchronize()
        return 0
    if args.kernel_only == "rowops":  # the layer's fused row ops at cfg2/cfg3 size (B8 T1568 H12 D64)
        from mlx_vit_b200.rowops import conv_silu, gated_rmsnorm
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        xr = torch.randn(B, T, H * D, generator=gen, device=dev).to(torch.bfloat16).requires_grad_(True)
        w = torch.randn(H * D, 1, 4, generator=gen, device=dev).requires_grad_(True)
        bias = torch.zeros(H * D, device=dev, requires_grad=True)
        o = torch.randn(B, T, H, D, generator=gen, device=dev).to(torch.bfloat16).requires_grad_(True)
        gt = torch.randn_like(o).requires_grad_(True)
        rw = torch.ones(D, device=dev, requires_grad=True)
        for _ in range(args.warmup + args.steps):
            y = conv_silu(xr, w, bias, H, D, True, D ** -0.5)
            z = gated_rmsnorm(o, gt, rw)
            torch.autograd.backward([y, z], [torch.ones_like(y), torch.ones_like(z)])
        torch.cuda.synchronize()
        return 0
    Bk = 2 if args.small else B  # --small: a case for multi-pass ncu captures (~100 MB resident)
    inp = make_inputs_torch(Bk, T, H, D, seed=1234, device=dev, dtype=torch.bfloat16, state_std=0.1)
    q, k, v, g, beta, S0, do, dst = (inp[n] for n in ("q", "k", "v", "g", "beta", "state", "do", "dst"))
    _, _, cs = kda_forward(q, k, v, g, beta, S0, CHUNK, save_states=True)
    if args.kernel_only == "gated":  # the fused-gate calls, reference gate init (A in [1, 16])
        from mlx_vit_b200.kda import kda_forward_gated, kda_backward_gated
        gen = torch.Generator(device=dev)
        gen.manual_seed(99)
        f = torch.randn(Bk, T, H, D, generator=gen, device=dev).to(torch.bfloat16)
        bl = torch.randn(Bk, T, H, generator=gen, device=dev).to(torch.bfloat16)
        A_log = torch.log(torch.rand(H, generator=gen, device=dev) * 15 + 1)
        dtb = torch.zeros(H * D, device=dev)
        for _ in range(args.warmup + args.steps):
            _, _, sg = kda_forward_gated(q, k, v, f, A_log, dtb, bl, S0, CHUNK, save_states=True)
            kda_backward_gated(q, k, v, f, A_log, dtb, bl, S0, sg, do, dst, CHUNK)
        torch.cuda.synchronize()
        return 0
    for _ in range(args.warmup + args.steps):
        if args.kernel_only in ("fwd", "both"):
            kda_forward(q, k, v, g, beta, S0, CHUNK, save_states=args.kernel_only == "both")
        if args.kernel_only in ("bwd", "both"):
            kda_backward(q, k, v, g, beta, S0, cs, do, dst, CHUNK)
    torch.cuda.synchronize()
    return 0


def run_cfg3(args, rank, world, local_rank, steps=None):
    """cfg3: full NoPE-GDN video model training step (12 KDA blocks, width 768, 12 x 64 heads,
    MLP 3072, tubelet 2x16x16, 400 classes), random init, bf16 autocast, 8 clips [16, 224, 224, 3]
    ~ U[0, 1] per GPU with random labels, data parallel over NCCL (torch DDP gradient
    all-reduce).  A step is forward + loss + backward + AdamW step; timed with CUDA events, max
    over ranks.  The KDA kernels' share of a step comes from one torch-profiler pass outside
    the timed region."""
    import torch
    import torch.nn.functional as F
    from mlx_vit_b200 import _lib
    from mlx_vit_b200.nope_gdn import NoPEGDNVideo
    from mlx_vit_b200.shard import max_over_ranks
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    torch.manual_seed(1234)  # same initial weights on every rank
    model = NoPEGDNVideo().to(dev)
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local_rank],
                                                          gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99 + rank)
    clips = torch.rand(8, 16, 224, 224, 3, generator=gen, device=dev)
    labels = torch.randint(0, 400, (8,), generator=gen, device=dev)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = F.cross_entropy(model(clips).float(), labels)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    steps = steps or args.steps
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    L0 = _lib.lib().kda_launch_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        e0.record()
        for _ in range(steps):
            loss = step()
        e1.record()
        torch.cuda.synchronize()
    launches = _lib.lib().kda_launch_counter() - L0
    total = max_over_ranks(e0.elapsed_time(e1), dev)
    ms = total / steps
    share = None
    # every rank runs the profiled step (DDP's all-reduce needs all of them); rank 0 records it
    import contextlib
    from torch.profiler import profile, ProfilerActivity
    with (profile(activities=[ProfilerActivity.CUDA]) if rank == 0 else contextlib.nullcontext()) as prof:
        step()
        torch.cuda.synchronize()
    if rank == 0:
        kda_us = all_us = 0.0
        for ev in prof.key_averages():
            t = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0.0)
            if ev.device_type is not None and "CUDA" in str(ev.device_type):
                all_us += t
                if "kda_" in ev.key:
                    kda_us += t
        share = round(kda_us / all_us, 4) if all_us else None
    if rank != 0:
        return None
    return {"metric": "NoPE-GDN video training step clips/s (cfg3)", "value": round(8 * world / (ms / 1e3), 2),
            "unit": "clips/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic clips U[0,1], random labels, random-init weights",
            "config": {"workload": "cfg3: 12 KDA blocks, width 768, 12x64 heads, MLP 3072, tubelet 2x16x16, "
                                   "400 classes, 8 clips x 16x224x224x3 per GPU (T = 1568 tokens)",
                       "parallelism": f"ddp x{world} (NCCL all-reduce)", "optimizer": "AdamW (fused)",
                       "l2": "inputs and activations far larger than L2"},
            "kda_share_of_gpu_time": share, "loss": round(float(loss), 4),
            "gpu_launches": int(launches), "clocks": clk.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-cfg3", action="store_true", help="leave out the nested config-3 leg")
    ap.add_argument("--small", action="store_true", help="with --kernel-only: B = 2 instead of 8")
    ap.add_argument("--workload", choices=("cfg2", "cfg3"), default="cfg2",
                    help="cfg2: the KDA op (the headline line); cfg3: full-model DP training step")
    ap.add_argument("--kernel-only", choices=("fwd", "bwd", "both", "stream", "gated", "recurrent", "rowops"),
                    default=None,
                    help="profiling driver: run only the kda_fwd/kda_bwd launches (steps+warmup "
                         "times), no timing, no e2e, no JSON line")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return 0
        v, cores, sample, tsec = cpu_reference(args.steps, args.warmup)
        line = {"metric": METRIC, "value": round(v, 1), "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tsec * 1e3, 2),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded; BASELINE config-2 distributions)",
                "impl": "reference",
                "config": {"workload": "cfg2: chunkwise KDA fwd+VJP, B8 H12 T1568 dk=dv=64 "
                                       "chunk64 (CPU sample)", "B": B, "H": H, "T": T, "D": D},
                "cpu_baseline": {"value": round(v, 1), "unit": UNIT, "cores": cores, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "MLX (the reference's runtime) is not installable here; the reference's "
                        "compiled path is timed as its numpy restatement (oracle/kda_oracle.py)"}
        print(json.dumps(line))
        return 0

    import torch
    if args.kernel_only:
        return kernel_only(args)
    if world > 1:
        import torch.distributed as dist
        import datetime
        # a short collective timeout: a rank that falls out ends the others' next collective
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
    line = run_cfg3(args, rank, world, local_rank) if args.workload == "cfg3" else run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
