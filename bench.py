"""Benchmark of the Mamba-3 scan hot path on B200.

Headline workload (one "step"): the raw SISO scan op ``ssm_scan_siso`` forward at long
context, bf16 I/O: B=16, H=64, P=64, D=128, L=32768 (x, B, C ~ N(0,1); dt =
clamp(softplus(N(-3, 0.5)), 1e-3, 0.1); A = -exp(U(0, ln 16)) per head; ADT = A dt;
trap = sigmoid(N(0,1)) passed as the op's logit; B and C rotated by RoPE with angles
cumsum(dt) * 10000^(-2i/D) on the first D/2 dims). Synthetic inputs, seeded per rank.
The batch is sharded across ranks (one process per GPU, torchrun), so the total work is
fixed as N grows; no collective runs inside the scan.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. ``value`` = tokens (B*L positions, all heads) per second
for the whole job, timed on the device with CUDA events (max over ranks); ``e2e`` is the
same metric through the public API with the inputs copied from pinned host memory and y
copied back every step (batch slices pipelined so that the copies in and out overlap);
``roofline`` relates the scan kernel's algorithmic bytes to the measured HBM copy
bandwidth; ``cpu_baseline`` times the fp32 C restatement of the reference's CPU loop on a
bounded sample (rank 0, N=1).
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mamba3-ssm_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

C5 = dict(batch=16, seqlen=32768, nheads=64, headdim=64, dstate=128)
METRIC = "scan tokens/s (SISO scan fwd, B=16 H=64 P=64 D=128 L=32768, bf16)"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def algorithmic_bytes_per_unit(e=2, P=64, D=128):
    """Bytes one (b, l, h) position must move: x, y (P each), B, C (D each) in the I/O
    dtype, plus ADT, DT, trap in fp32."""
    return e * (2 * P + 2 * D) + 12


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ----------------------------------------------------------------------------------
# multi-rank helpers (one process per GPU; the scan needs no exchange)
# ----------------------------------------------------------------------------------
def shard(total, world, rank):
    """Contiguous share of `total` batch rows for `rank`: (first row, rows)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def max_over_ranks(values, dist=None, device=None):
    """Element-wise max of a list of floats over all ranks (the job's time is the slowest
    rank's). With no process group the values are returned unchanged."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


# ----------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, gpu_ids):
        self.idx = ",".join(str(i) for i in gpu_ids)
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.idx, "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except (OSError, ValueError):
            self.proc = None
            return
        # nvidia-smi's first query of the throttle reasons stalls the GPU for ~0.1 s: let it
        # land before the timed region starts
        t0 = time.time()
        while not self.lines and time.time() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.05)
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.th.join(timeout=2)
        sm, mx, mem, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
            if len(f) > 9:
                try:
                    mem.append(float(f[9]))
                except ValueError:
                    pass
        if not sm:
            return None
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
               "samples": len(sm)}
        if mem:
            out["mem_mhz"] = statistics.median(mem)
        return out


# ----------------------------------------------------------------------------------
# inputs
# ----------------------------------------------------------------------------------
def make_inputs(batch, L, H, P, D, device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    bf = torch.bfloat16
    x = torch.empty(batch, L, H, P, dtype=bf, device=device)
    Bm = torch.empty(batch, L, H, D, dtype=bf, device=device)
    Cm = torch.empty(batch, L, H, D, dtype=bf, device=device)
    dt = F.softplus(torch.randn(batch, L, H, generator=g, device=device) * 0.5 - 3.0).clamp(1e-3, 0.1)
    A = -torch.exp(torch.rand(H, generator=g, device=device) * math.log(16.0))
    ADT = (A * dt).contiguous()
    trap = torch.sigmoid(torch.randn(batch, L, H, generator=g, device=device))
    Dw = torch.randn(H, generator=g, device=device) * 0.5 + 1.0
    S = D // 4
    theta = 10000.0 ** (-2.0 * torch.arange(S, device=device, dtype=torch.float32) / D)
    for b in range(batch):
        x[b] = torch.randn(L, H, P, generator=g, device=device).to(bf)
        ang = torch.cumsum(dt[b], dim=0).unsqueeze(-1) * theta  # (L, H, S)
        c, s = torch.cos(ang), torch.sin(ang)
        for dst in (Bm, Cm):
            v = torch.randn(L, H, D, generator=g, device=device)
            v1, v2 = v[..., 0:2 * S:2].clone(), v[..., 1:2 * S:2].clone()
            v[..., 0:2 * S:2] = v1 * c - v2 * s
            v[..., 1:2 * S:2] = v1 * s + v2 * c
            dst[b] = v.to(bf)
    return x, Bm, Cm, ADT, dt.contiguous(), trap.contiguous(), Dw


# ----------------------------------------------------------------------------------
# CPU baseline: fp32 C restatement of the reference loop, bounded sample
# ----------------------------------------------------------------------------------
def cpu_sample(L_sample, nb=1, H=64, P=64, D=128, seed=7):
    import numpy as np
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((nb, L_sample, H, P), dtype=np.float32)
    Bm = rng.standard_normal((nb, L_sample, H, D), dtype=np.float32)
    Cm = rng.standard_normal((nb, L_sample, H, D), dtype=np.float32)
    dt = np.clip(np.log1p(np.exp(rng.normal(-3, 0.5, (nb, L_sample, H)))), 1e-3, 0.1).astype(np.float32)
    A = -np.exp(rng.uniform(0, np.log(16), H)).astype(np.float32)
    trap = (1 / (1 + np.exp(-rng.standard_normal((nb, L_sample, H))))).astype(np.float32)
    return x, Bm, Cm, (A * dt).astype(np.float32), dt, trap, np.ones(H, np.float32)


def cpu_baseline(target_s=12.0, L_s=4096):
    """Time the fp32 C restatement of the reference loop on all host cores on a bounded
    sample of the long-context workload: one batch row x 64 heads x L_s positions (about
    0.4 GB of host arrays), run repeatedly until about target_s seconds have passed (the
    per-position cost of the loop does not depend on the position). Returns
    (baseline dict, (L_s, reps per step of about 2 s))."""
    from oracle import cpu_ref
    cores = cpu_ref.max_threads()
    args = cpu_sample(L_s)
    cpu_ref.siso_fwd(*args, nthreads=cores)  # warm-up (page-in, thread pool)
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_ref.siso_fwd(*args, nthreads=cores)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    tok_s = reps * L_s / dt
    per_2s = max(1, int(round(2.0 * reps / dt)))
    return {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"fp32 C restatement of the reference loop (oracle/scan_ref.c), OpenMP over (b,h); "
                      f"1 batch row x 64 heads x {L_s} positions (P=64, D=128) of the long-context workload, "
                      f"run {reps} times in {dt:.1f} s"}, (L_s, per_2s)


def check_units(inputs, y, units):
    """Max rel error (max|y - ref| / max|ref|) of the kernel's y on a few (b, h) units
    against a float64 restatement of the scan recurrence run on the host here (the
    exponential-trapezoidal update of the reference loop, ops.py:166-175):
    h_t = e^{ADT_t} h_{t-1} + dt_t ((1 - tr_t) x_t B_t + tr_t (x_t B_t + x_{t-1} B_{t-1}) / 2),
    y_t = h_t C_t + D x_t, tr = sigmoid(trap). Independent of the kernels."""
    import numpy as np
    x, Bm, Cm, ADT, DT, trap, Dw = inputs
    sel = lambda t: np.stack([t[b, :, h].double().cpu().numpy() for b, h in units], axis=1)  # noqa: E731
    xs, bs, cs = sel(x), sel(Bm), sel(Cm)          # (L, n, P|D)
    a = np.exp(sel(ADT))                            # (L, n)
    dt = sel(DT)
    tr = 1.0 / (1.0 + np.exp(-sel(trap)))
    dsk = np.array([float(Dw[h]) for _, h in units])
    n, P, D = xs.shape[1], xs.shape[2], bs.shape[2]
    h = np.zeros((n, P, D))
    bxp = np.zeros((n, P, D))
    ref = np.empty_like(xs)
    for t in range(xs.shape[0]):
        bx = xs[t][:, :, None] * bs[t][:, None, :]
        w1 = (dt[t] * (1.0 - 0.5 * tr[t]))[:, None, None]
        w2 = (dt[t] * 0.5 * tr[t])[:, None, None]
        h = a[t][:, None, None] * h + w1 * bx + w2 * bxp
        ref[t] = np.einsum("npd,nd->np", h, cs[t]) + dsk[:, None] * xs[t]
        bxp = bx
    got = sel(y)
    return float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))


def workload_config(world):
    return {"workload": "raw SISO scan op forward, long context (ssm_scan_siso)", "batch": C5["batch"],
            "seq_len": C5["seqlen"], "nheads": C5["nheads"], "headdim": C5["headdim"], "d_state": C5["dstate"],
            "parallelism": f"batch-sharded x{world}", "l2": "inputs (26 GB) larger than L2"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    from oracle import cpu_ref
    cores = cpu_ref.max_threads()
    # one step = the sample run enough times for about 2 s of CPU work
    base, (L_s, reps) = cpu_baseline(target_s=4.0)
    sample = cpu_sample(L_s)
    for _ in range(args.warmup):
        cpu_ref.siso_fwd(*sample, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps * reps):
        cpu_ref.siso_fwd(*sample, nthreads=cores)
    el = time.perf_counter() - t0
    v = args.steps * reps * L_s / el
    base["value"] = v
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": workload_config(world),
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------
# secondary figures (one GPU): long-context forward + backward, and LM decode
# ----------------------------------------------------------------------------------
def measure_fwd_bwd(inputs, steps=2):
    """ssm_scan_siso forward + backward through autograd on the long-context inputs."""
    from mamba3_ssm import ssm_scan_siso
    x, Bm, Cm, ADT, DT, trap, Dw = inputs
    leaves = [t.detach().requires_grad_(True) for t in (x, Bm, Cm, ADT, DT, trap, Dw)]
    dy = torch.randn_like(x)
    for _ in range(1):
        ssm_scan_siso(*leaves).backward(dy)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        for t in leaves:
            t.grad = None
        ssm_scan_siso(*leaves).backward(dy)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    tokens = x.shape[0] * x.shape[1]
    return {"value": tokens / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": steps,
            "what": "ssm_scan_siso forward + backward (autograd) on the same workload"}


def _state_bytes(mixer, batch):
    """fp32 decode-state bytes of one layer: angle (B,H,S) + ssm and bx (B,H,D) MIMO or
    (B,H,P,D) SISO."""
    per = mixer.d_state if mixer.is_mimo else mixer.headdim * mixer.d_state
    return batch * mixer.nheads * (mixer.num_rope_angles + 2 * per) * 4


def measure_decode(dev, steps=48, batch=256, prefill=16):
    """Greedy decode of the medium preset (d_model 1536, 20 layers, MIMO rank 4, d_state 64,
    headdim 64, vocab 50000), bf16, batch 256, random-init weights, uniform random prompt
    ids, three ways: MambaLMHeadModel.step (block.py:110-139 interface, one launch per op),
    the same step replayed as one CUDA graph (DecodeGraph), and the fused step kernel alone
    (m3_mimo_step per layer, cycling the 20 layers' caches so the state exceeds L2)."""
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=1536, n_layer=20, vocab_size=50000,
                      ssm_cfg=dict(d_state=64, expand=2, headdim=64, is_mimo=True, mimo_rank=4))
    model = MambaLMHeadModel(cfg, device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    ids = torch.randint(0, 50000, (batch, prefill), device=dev, generator=g)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    with torch.no_grad():
        # (1) eager step()
        cache = model.allocate_inference_cache(batch)
        for t in range(prefill):
            logits, cache = model.step(ids[:, t], cache)
        tok = logits.argmax(-1)
        for _ in range(3):
            logits, cache = model.step(tok, cache)
            tok = logits.argmax(-1)
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(steps):
            logits, cache = model.step(tok, cache)
            tok = logits.argmax(-1)
        e1.record()
        torch.cuda.synchronize()
        ms_eager = e0.elapsed_time(e1) / steps
        del cache, logits
        # (2) CUDA-graph replay of the whole step (greedy argmax inside the graph)
        dg = model.decode_graph(batch, greedy=True)
        for t in range(prefill):
            dg.feed(ids[:, t])
        for _ in range(3):
            dg.next()
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(steps):
            dg.next()
        e1.record()
        torch.cuda.synchronize()
        ms_graph = e0.elapsed_time(e1) / steps
        del dg
        # (3) the fused step kernel alone, one launch per layer
        mixers = [blk.mixer for blk in model.layers]
        u = torch.randn(batch, cfg.d_model, device=dev, dtype=torch.bfloat16)
        zs = [m.in_proj(u).contiguous() for m in mixers]
        caches = [m.allocate_inference_cache(batch) for m in mixers]
        ys = [torch.empty(batch, m.d_inner, device=dev, dtype=torch.bfloat16) for m in mixers]
        def sweep():
            for m, z, c, y in zip(mixers, zs, caches, ys):
                m._fused_step(z, *c, *c, y)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                sweep()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()  # replayed, so host-side binding cost is not timed
        with torch.cuda.graph(graph):
            sweep()
        graph.replay()
        torch.cuda.synchronize()
        kreps = 10
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(kreps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us_kernel = e0.elapsed_time(e1) * 1e3 / (kreps * len(mixers))
        del graph
    m0 = mixers[0]
    kbytes = (2 * _state_bytes(m0, batch) + zs[0].numel() * zs[0].element_size()
              + ys[0].numel() * ys[0].element_size())
    k_gbs = kbytes / (us_kernel * 1e-6) / 1e9
    peak = peaks()[0]
    state_bytes = 20 * 2 * _state_bytes(m0, batch)
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    del model, caches, zs, ys
    torch.cuda.empty_cache()
    return {"value": batch / (ms_graph / 1e3), "unit": "tokens/s", "ms_per_step": ms_graph,
            "eager_step": {"value": batch / (ms_eager / 1e3), "ms_per_step": ms_eager},
            "steps": steps, "batch": batch, "layers": 20, "bytes_per_step_min": state_bytes + weight_bytes,
            "step_kernel": {"us_per_launch": us_kernel, "bytes_per_launch": kbytes, "achieved_gbs": k_gbs,
                            "peak_gbs": peak, "frac": k_gbs / peak,
                            "what": "m3_mimo_step, one layer at batch 256 (in-place state), 20 layers' "
                                    "caches cycled, replayed from a CUDA graph"},
            "what": "greedy decode, medium preset (d_model 1536, 20 layers, MIMO R=4), bf16, batch 256, "
                    "after a 16-token prefill; value = DecodeGraph replay, eager_step = "
                    "MambaLMHeadModel.step"}


def _time(fn, steps, warm=2):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def measure_mimo(dev, steps=10):
    """MIMO at the layer configuration the reference's tests use for bf16 MIMO (d_model 256,
    H=16, P=32, D=64, R=4, batch 8 x 2048 tokens): the raw op ssm_scan_mimo forward on the
    layer's operand types (x bf16, B/C fp32) with its HBM roofline, and Mamba3.forward +
    backward through the whole layer (random-init weights, synthetic activations)."""
    from mamba3_ssm import Mamba3, ssm_scan_mimo
    torch.manual_seed(0)
    Bn, L, H, P, D, R = 8, 2048, 16, 32, 64, 4
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    x = torch.randn(Bn, L, H, P, device=dev, generator=g).to(torch.bfloat16)
    Bm = torch.randn(Bn, L, R, H, D, device=dev, generator=g)
    Cm = torch.randn(Bn, L, R, H, D, device=dev, generator=g)
    dt = F.softplus(torch.randn(Bn, L, H, device=dev, generator=g) * 0.5 - 3.0).clamp(1e-3, 0.1)
    ADT = (-torch.exp(torch.rand(H, device=dev, generator=g) * math.log(16.0)) * dt).contiguous()
    trap = torch.randn(Bn, L, H, device=dev, generator=g)
    Dw = torch.ones(H, device=dev)
    mx = torch.randn(H, R, P, device=dev, generator=g) * 0.3 + 0.25
    mo = torch.randn(H, R, P, device=dev, generator=g) * 0.3 + 0.25
    with torch.no_grad():
        op_ms = _time(lambda: ssm_scan_mimo(x, Bm, Cm, ADT, dt, trap, Dw, mx, mo), steps)
    op_bytes = Bn * L * H * (2 * 2 * P + 2 * 4 * R * D + 12)
    peak = peaks()[0]
    layer = Mamba3(d_model=256, d_state=64, expand=2, headdim=32, is_mimo=True, mimo_rank=4,
                   device=dev, dtype=torch.bfloat16)
    u = torch.randn(Bn, L, 256, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(Bn, L, 256, device=dev, generator=g).to(torch.bfloat16)

    def fb():
        for p_ in layer.parameters():
            p_.grad = None
        u.grad = None
        layer(u).backward(dy)
    fb_ms = _time(fb, steps)
    with torch.no_grad():
        f_ms = _time(lambda: layer(u), steps)
    del layer, u, dy, x, Bm, Cm
    torch.cuda.empty_cache()
    tok = Bn * L
    return {"op_fwd": {"ms": op_ms, "tokens_per_s": tok / (op_ms / 1e3), "bytes": op_bytes,
                       "achieved_gbs": op_bytes / (op_ms / 1e3) / 1e9, "frac_hbm": op_bytes / (op_ms / 1e3) / 1e9 / peak,
                       "what": "ssm_scan_mimo forward, x bf16, B/C fp32 (B,L,R,H,D), R=4 H=16 P=32 D=64, 8 x 2048"},
            "layer_fwd": {"ms": f_ms, "tokens_per_s": tok / (f_ms / 1e3)},
            "layer_fwd_bwd": {"ms": fb_ms, "tokens_per_s": tok / (fb_ms / 1e3)},
            "what": "Mamba3 MIMO layer (d_model 256, R=4, bf16), batch 8 x 2048 tokens"}


def measure_lm_forward(dev, steps=5):
    """MambaLMHeadModel forward at the SISO LM preset (d_model 1024, 16 layers, H=32, P=64,
    D=64, vocab 50000), bf16, batch 32 x 512 tokens, random-init weights, uniform ids;
    reported against the measured bf16 tensor peak (the forward is GEMM-bound)."""
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=1024, n_layer=16, vocab_size=50000,
                      ssm_cfg=dict(d_state=64, expand=2, headdim=64))
    model = MambaLMHeadModel(cfg, device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    ids = torch.randint(0, 50000, (32, 512), device=dev, generator=g)
    with torch.no_grad():
        ms = _time(lambda: model(ids), steps)
    d_in_proj = model.layers[0].mixer.in_proj.weight.shape[0]
    flops_tok = 2 * 16 * (1024 * d_in_proj + 2048 * 1024) + 2 * 1024 * model.vocab_size
    tflops = flops_tok * ids.numel() / (ms / 1e3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk = float(json.load(f).get("bf16_tflops", 1590.0))
    except (OSError, ValueError):
        tpk = 1590.0
    del model
    torch.cuda.empty_cache()
    return {"ms": ms, "tokens_per_s": ids.numel() / (ms / 1e3), "gemm_tflops": tflops,
            "frac_bf16_peak": tflops / tpk, "flops_per_token": flops_tok,
            "what": "MambaLMHeadModel.forward, SISO preset d_model 1024 x 16 layers, bf16, 32 x 512 tokens"}


def measure_lm_dp(dev, world, rank, pg, steps=4, dec_steps=32):
    """The two LM workloads data-parallel over the job's ranks: each rank holds a full
    weight replica (same seed) and its share of the batch; no collective runs inside a
    timed region, which is bracketed by barriers and taken as the max over ranks.
      c3_lm_forward   MambaLMHeadModel.forward, SISO preset (d_model 1024, 16 layers, vocab
                      50000), bf16, global batch 32 x 512 tokens;
      c4_decode       greedy decode of the MIMO preset (d_model 1536, 20 layers, R=4, vocab
                      50000), bf16, global batch 256, one whole step replayed as a CUDA
                      graph after a 16-token prefill;
      c4_step_kernel  the fused decode-step kernel alone (20 layers at the rank's batch
                      share, caches cycled), the state-bound part of the decode step.
    Full-LM decode carries the replicated weights (761 MB per step on every GPU), so it
    cannot scale like the state-bound step kernel; both are reported."""
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def barrier():
        if pg is not None:
            pg.barrier()

    def timed(fn, n):
        torch.cuda.synchronize()
        barrier()
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        (ms,) = max_over_ranks([e0.elapsed_time(e1) / n], pg, dev)
        return ms

    out = {}
    _, b3 = shard(32, world, rank)
    torch.manual_seed(0)
    cfg3 = MambaConfig(d_model=1024, n_layer=16, vocab_size=50000, ssm_cfg=dict(d_state=64, expand=2, headdim=64))
    m3 = MambaLMHeadModel(cfg3, device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    ids = torch.randint(0, 50000, (b3, 512), device=dev, generator=g)
    with torch.no_grad():
        for _ in range(2):
            m3(ids)
        ms3 = timed(lambda: m3(ids), steps)
    out["c3_lm_forward"] = {"value": 32 * 512 / (ms3 / 1e3), "unit": "tokens/s", "ms_per_step": ms3,
                            "batch_per_rank": b3, "global_batch": 32, "seq_len": 512, "steps": steps}
    del m3, ids
    torch.cuda.empty_cache()

    _, b4 = shard(256, world, rank)
    torch.manual_seed(0)
    cfg4 = MambaConfig(d_model=1536, n_layer=20, vocab_size=50000,
                       ssm_cfg=dict(d_state=64, expand=2, headdim=64, is_mimo=True, mimo_rank=4))
    m4 = MambaLMHeadModel(cfg4, device=dev, dtype=torch.bfloat16).eval()
    prompt = torch.randint(0, 50000, (b4, 16), device=dev, generator=g)
    with torch.no_grad():
        dg = m4.decode_graph(b4, greedy=True)
        for t in range(16):
            dg.feed(prompt[:, t])
        for _ in range(3):
            dg.next()
        ms4 = timed(dg.next, dec_steps)
        del dg
        mixers = [blk.mixer for blk in m4.layers]
        u = torch.randn(b4, cfg4.d_model, device=dev, dtype=torch.bfloat16, generator=g)
        zs = [mx.in_proj(u).contiguous() for mx in mixers]
        caches = [mx.allocate_inference_cache(b4) for mx in mixers]
        ys = [torch.empty(b4, mx.d_inner, device=dev, dtype=torch.bfloat16) for mx in mixers]

        def sweep():
            for mx, z, c, y in zip(mixers, zs, caches, ys):
                mx._fused_step(z, *c, *c, y)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                sweep()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()  # replayed, so the host-side binding cost is not timed
        with torch.cuda.graph(graph):
            sweep()
        graph.replay()
        us_k = timed(graph.replay, 10) * 1e3 / len(mixers)
        del graph
    kbytes = (2 * _state_bytes(mixers[0], b4) + zs[0].numel() * zs[0].element_size()
              + ys[0].numel() * ys[0].element_size())
    peak = peaks()[0]
    out["c4_decode"] = {"value": 256 / (ms4 / 1e3), "unit": "tokens/s", "ms_per_step": ms4, "batch_per_rank": b4,
                        "global_batch": 256, "steps": dec_steps,
                        "what": "whole greedy decode step (CUDA graph): embedding, 20 layers, norm_f, lm_head, argmax"}
    out["c4_step_kernel"] = {"value": 256 / (len(mixers) * us_k * 1e-6), "unit": "tokens/s", "us_per_launch": us_k,
                             "batch_per_rank": b4, "bytes_per_launch": kbytes,
                             "achieved_gbs_per_gpu": kbytes / (us_k * 1e-6) / 1e9,
                             "frac_hbm_per_gpu": kbytes / (us_k * 1e-6) / 1e9 / peak,
                             "what": "fused decode-step kernel only (m3_mimo_step), 20 layers per token step replayed "
                                     "from a CUDA graph; value = tokens/s of the job if a decode step were these 20 "
                                     "launches"}
    # weak scaling of the same kernel: the full batch of 256 on every rank
    with torch.no_grad():
        if world > 1:
            uw = torch.randn(256, cfg4.d_model, device=dev, dtype=torch.bfloat16, generator=g)
            zw = [mx.in_proj(uw).contiguous() for mx in mixers]
            cw = [mx.allocate_inference_cache(256) for mx in mixers]
            yw = [torch.empty(256, mx.d_inner, device=dev, dtype=torch.bfloat16) for mx in mixers]

            def sweep_w():
                for mx, z, c, y in zip(mixers, zw, cw, yw):
                    mx._fused_step(z, *c, *c, y)
            with torch.cuda.stream(side):
                for _ in range(3):
                    sweep_w()
            torch.cuda.current_stream(dev).wait_stream(side)
            gw = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gw):
                sweep_w()
            gw.replay()
            us_w = timed(gw.replay, 10) * 1e3 / len(mixers)
            del gw, zw, cw, yw, uw
            out["c4_step_kernel_weak"] = {"value": 256 * world / (len(mixers) * us_w * 1e-6), "unit": "tokens/s",
                                          "us_per_launch": us_w, "batch_per_rank": 256, "global_batch": 256 * world,
                                          "scaling": "weak",
                                          "what": "the same kernel with the full batch of 256 on every rank"}
    del m4, zs, caches, ys, u
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the forward+backward and decode figures")
    ap.add_argument("--no-check", action="store_true", help="skip the host check of the timed output")
    ap.add_argument("--no-sustained", action="store_true", help="skip the ~2 s sustained run")
    ap.add_argument("--no-lm", action="store_true", help="skip the data-parallel LM forward / decode figures")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the global batch (profiling runs on a smaller case)")
    ap.add_argument("--fwd-bwd-only", action="store_true",
                    help="only the ssm_scan_siso forward + backward figure (profiling the backward)")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the decode figure (profiling the decode step)")
    ap.add_argument("--mimo-only", action="store_true",
                    help="only the MIMO op / layer figures (profiling the MIMO kernels)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    from mamba3_ssm import ssm_scan_siso
    from mamba3_ssm import _lib
    _lib.load()
    if args.decode_only:
        r = measure_decode(dev)
        if rank == 0:
            print(json.dumps({"decode": r, "timeouts": _lib.device_timeouts(reset=True)}))
        return
    if args.mimo_only:
        r = measure_mimo(dev)
        if rank == 0:
            print(json.dumps({"mimo": r, "timeouts": _lib.device_timeouts(reset=True)}))
        return

    if args.batch:
        C5["batch"] = args.batch
    Bt, L, H, P, D = C5["batch"], C5["seqlen"], C5["nheads"], C5["headdim"], C5["dstate"]
    _, Bl = shard(Bt, world, rank)
    x, Bm, Cm, ADT, DT, trap, Dw = make_inputs(Bl, L, H, P, D, dev, 1234 + rank)
    torch.cuda.synchronize()
    if args.fwd_bwd_only:
        r = measure_fwd_bwd((x, Bm, Cm, ADT, DT, trap, Dw), steps=args.steps)
        if rank == 0:
            print(json.dumps({"fwd_bwd": r, "batch": Bl, "timeouts": _lib.device_timeouts(reset=True)}))
        return

    def barrier():
        if pg is not None:
            pg.barrier()

    def step():
        return ssm_scan_siso(x, Bm, Cm, ADT, DT, trap, Dw)

    # untimed warm-up: at least W steps and at least ~1 s of work, so that the first timed
    # step does not see the GPU's clocks still ramping up from idle
    n_warm, t_w = 0, time.time()
    while n_warm < max(3, args.warmup) or time.time() - t_w < 1.0:
        step()
        n_warm += 1
        if n_warm % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    n_warm, = max_over_ranks([n_warm], pg, dev)
    K = args.steps
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    t_beg, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # every rank's GPU, named by UUID (nvidia-smi indices need not match CUDA ordinals)
    uid = str(torch.cuda.get_device_properties(dev).uuid)
    uid = uid if uid.startswith("GPU-") else "GPU-" + uid
    uids = [uid]
    if pg is not None:
        uids = [None] * world
        pg.all_gather_object(uids, uid)
    sampler = ClockSampler(uids) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier()
    torch.cuda.synchronize()
    t_beg.record()
    for i in range(K):
        evs[i][0].record()
        y = step()
        evs[i][1].record()
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    if _lib.device_timeouts(reset=True):
        raise RuntimeError("a bounded inter-warp wait gave up during the timed region; outputs invalid")
    total_ms = t_beg.elapsed_time(t_end)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    total_ms, kern_ms = max_over_ranks([total_ms, kern_ms], pg, dev)

    # the timed output, checked on two (b, h) units of this rank against a float64
    # recurrence on the host (first and last unit of the shard)
    check = None
    if not args.no_check:
        units = [(0, 0), (Bl - 1, H - 1)]
        err = check_units((x, Bm, Cm, ADT, DT, trap, Dw), y, units)
        (err,) = max_over_ranks([err], pg, dev)
        check = {"max_rel_err": err, "bar": 2e-2, "ok": err < 2e-2,
                 "what": "y of the last timed step on units (b, h) = (0, 0) and (last, last) of every rank's "
                         "shard against a float64 host recurrence, max|y - ref| / max|ref|"}

    # a sustained run of at least ~2 s after the timed region, with its own clock record
    # (K steps of the timed region can be well under a second)
    sustained = None
    if not args.no_sustained:
        n_s = max(K, int(math.ceil(2000.0 / max(total_ms / K, 1e-3))))
        sampler2 = ClockSampler(uids) if rank == 0 else None
        if sampler2:
            sampler2.start()
        barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(n_s):
            step()
        s1.record()
        torch.cuda.synchronize()
        barrier()
        clk2 = sampler2.stop() if sampler2 else None
        (s_ms,) = max_over_ranks([s0.elapsed_time(s1)], pg, dev)
        sustained = {"steps": n_s, "seconds": s_ms / 1e3, "ms_per_step": s_ms / n_s,
                     "value": Bt * L / (s_ms / n_s / 1e3), "clocks": clk2,
                     "what": "the same step repeated for ~2 s right after the timed region"}
    ms_step = total_ms / K
    tokens = Bt * L
    value = tokens / (ms_step / 1e3)

    hbm, peak_kind = peaks()
    unit_bytes = algorithmic_bytes_per_unit()
    launch_bytes = unit_bytes * Bl * L * H
    achieved = launch_bytes / (kern_ms / 1e3) / 1e9
    tr = measured_traffic().get("siso_scan_fwd")
    traffic = tr["bytes_per_unit"] * Bl * L * H if tr else None

    # e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        hosts = []
        for t in (x, Bm, Cm, ADT, DT, trap):
            h_ = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h_.copy_(t)
            hosts.append(h_)
        y_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        h2d = sum(h.numel() * h.element_size() for h in hosts)
        d2h = y_host.numel() * y_host.element_size()
        Ke = min(K, 3)
        devs = (x, Bm, Cm, ADT, DT, trap)
        # Batch slices pipelined over three streams: inputs in on `cin`, the scan on the
        # current stream, y out on `cout`. PCIe is full duplex, so slice s's y copy-back
        # overlaps the later slices' (and the next step's) input copies; a slice's inputs
        # are overwritten only after the scan that read them has finished.
        nsl = 4 if Bl % 4 == 0 else 1
        rows = Bl // nsl
        slices = [slice(i * rows, (i + 1) * rows) for i in range(nsl)]
        main = torch.cuda.current_stream(dev)
        cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        read_done = [None] * nsl
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(main)
        cin.wait_stream(main)
        cout.wait_stream(main)
        for _ in range(Ke):
            for i, s in enumerate(slices):
                with torch.cuda.stream(cin):
                    if read_done[i] is not None:
                        cin.wait_event(read_done[i])
                    for d_, h_ in zip(devs, hosts):
                        d_[s].copy_(h_[s], non_blocking=True)
                    arrived = torch.cuda.Event()
                    arrived.record(cin)
                main.wait_event(arrived)
                yy = ssm_scan_siso(x[s], Bm[s], Cm[s], ADT[s], DT[s], trap[s], Dw)
                read_done[i] = torch.cuda.Event()
                read_done[i].record(main)
                with torch.cuda.stream(cout):
                    cout.wait_event(read_done[i])
                    y_host[s].copy_(yy, non_blocking=True)
                    yy.record_stream(cout)
        main.wait_stream(cin)
        main.wait_stream(cout)
        e1.record(main)
        torch.cuda.synchronize()
        barrier()
        (e_ms,) = max_over_ranks([e0.elapsed_time(e1) / Ke], pg, dev)
        h2d, d2h = max_over_ranks([h2d, d2h], pg, dev)  # equal shares: report the job total below
        e2e = {"value": tokens / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d * world),
               "d2h_bytes_per_step": int(d2h * world), "steps": Ke,
               "batch_slices": nsl}
        del hosts, y_host

    extra = {}
    if not args.no_extra and not args.no_lm:
        del y
        extra["lm_dp"] = measure_lm_dp(dev, world, rank, pg)
        y = None
    if world == 1 and not args.no_extra:
        extra["fwd_bwd"] = measure_fwd_bwd((x, Bm, Cm, ADT, DT, trap, Dw))
        del x, Bm, Cm, ADT, DT, trap, Dw
        y = None
        torch.cuda.empty_cache()
        extra["decode"] = measure_decode(dev)
        extra["mimo"] = measure_mimo(dev)
        extra["lm_forward"] = measure_lm_forward(dev)

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base, _ = cpu_baseline()

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
                "warmup": int(n_warm), "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": workload_config(world),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind,
                             "algorithmic_bytes_per_launch": launch_bytes, "kernel_ms": kern_ms},
                "cpu_baseline": base, "e2e": e2e, "gpu_launches": K, "clocks": clocks,
                "check": check, "sustained": sustained, "secondary": extra}
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
