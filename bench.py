"""Headline benchmark: Atlas scan fwd+bwd tokens/s at the 170M configuration.

One step = for each of the 12 layers the forward scan (B=8/GPU, T=8192, 12 heads x 64,
memory MLP 64->256->64, chunk 64, Omega 16, 5 Polar Express steps, pe_ste=False,
bf16 activations, fp32 carry), then the 12 backward scans in reverse layer order,
then (N > 1) the NCCL all-reduce of an fp32 gradient buffer of the model's exact
parameter count (atlas_jax/train.py:150-152).  Inputs are synthetic with the
BASELINE distributions (q,k,v ~ N(0,1) L2-normalised per head, sigmoid gates), one
independent set per layer; every layer's inputs (~420 MB) exceed the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  --impl reference times the CPU restatement of the
reference scan (oracle/, numpy) on the host cores on a bounded sample.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "atlas-jax_b200"))

CFG = dict(layers=12, B=8, T=8192, H=12, D=64, E=256, chunk=64, omega=16, ns_steps=5)
METRIC = "Atlas scan tokens/s fwd+bwd (170M cfg)"
# algorithmic FLOPs per token-head-layer (m = D, n = E = 4D, ns steps); recompute not counted
F_FWD = lambda D, ns: ns * 36 * D ** 3 + 40 * D ** 2   # noqa: E731
F_BWD = lambda D, ns: ns * 56 * D ** 3 + 80 * D ** 2   # noqa: E731
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch, from an ncu
# capture of the small case (1 layer, B=8, H=12, T=256).  Both kernels' traffic is
# per token-head (the backward's Newton-Schulz operand scratch, S_t and W_{t-1}; the
# forward's saved carries and outputs), so a full launch scales by token-heads.
NCU_TRAFFIC = {"tc_bwd_kernel": 61.30e9, "tc_fwd_kernel": 112.8e6}
NCU_TOKEN_HEADS = 8 * 256 * 12


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1400.0, 6650.0, "fallback"


CPU_SAMPLE = dict(B=1, H=12, T=128)  # two chunks per head: the cross-chunk carry path is in the sample


def cpu_baseline():
    """Times the oracle (numpy restatement of the reference scan, float32, BLAS on all
    host threads) fwd+bwd on one layer of B=1, H=12, T=128, D=64 (two chunks per head);
    returns full-model tokens/s (a full token passes 12 heads x 12 layers)."""
    import numpy as np
    from oracle import atlas_oracle as O
    c, smp = CFG, CPU_SAMPLE
    ins = O.make_inputs(smp["B"], smp["T"], smp["H"], c["D"], seed=0)
    st = O.lm_initial_state(smp["B"], smp["H"], c["D"], c["E"])
    t0 = time.perf_counter()
    y, _ = O.scan_forward(*ins, st, c["chunk"], c["omega"], c["ns_steps"])
    dy = np.ones_like(y)
    O.scan_backward(*ins, st, dy, None, c["chunk"], c["omega"], c["ns_steps"], dtype=np.float32)
    dt = time.perf_counter() - t0
    equiv_tokens = smp["B"] * smp["T"] * smp["H"] / (c["H"] * c["layers"])
    return equiv_tokens / dt, dt, os.cpu_count()


CPU_SAMPLE_TEXT = ("oracle numpy restatement (float32), fwd+bwd of 1 layer, B=1 H=12 T=128 (2 chunks) D=64 E=256, "
                   "scaled to 12 heads x 12 layers per token")


def reference_arm(args, rank):
    if rank != 0:
        return
    vals = []
    for i in range(args.warmup + args.steps):
        v, dt, cores = cpu_baseline()
        if i >= args.warmup:
            vals.append(v)
    v = sorted(vals)[len(vals) // 2]
    sample = CPU_SAMPLE_TEXT
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "170M scan (CPU sample)", **CFG},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


class Clocks:
    def __init__(self, path):
        self.path, self.proc = path, None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self, gpu_index):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9 or p[0] != str(gpu_index):
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def f32_mode(lib, L, dev, stream, sp, p_bf16, nws, ws, g, world, layers=2, reps=2, f32=True, pe_ste=0):
    """A variant of the headline scan: float32 activations (the reference's float32
    path, held to its float32 accuracy), or pe_ste=True (the straight-through Polar
    Express backward, memory_layer.py:74-76).  `layers` layers of fwd+bwd, one untimed
    pass, then `reps` timed passes; tokens/s of the 12-layer step implied by the
    per-layer time."""
    import torch
    c = CFG
    B, T, H, D, E = c["B"], c["T"], c["H"], c["D"], c["E"]
    p = L.AtlasScanParams(*[getattr(p_bf16, n) for n, _ in L.AtlasScanParams._fields_])
    p.act_dtype = L.ATLAS_F32 if f32 else L.ATLAS_BF16
    p.pe_ste = pe_ste
    act = torch.float32 if f32 else torch.bfloat16
    pp = ctypes.byref(p)
    if lib.atlas_scan_workspace_bytes(pp) > nws:
        return None
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    Ls = []
    for _ in range(layers):
        Ld = {n: torch.nn.functional.normalize(torch.randn(B, T, H, D, device=dev, generator=g), dim=-1).to(act)
              for n in ("q", "k", "v")}
        for n, mu in (("alpha", 3.0), ("eta", -3.0), ("theta", 1.0), ("gamma", 0.0)):
            Ld[n] = torch.sigmoid(mu + 0.5 * torch.randn(B, T, H, device=dev, generator=g))
        Ld["dy"] = (torch.randn(B, T, H, D, device=dev, generator=g) * 0.01).to(act)
        for n in ("y", "dq", "dk", "dv"):
            Ld[n] = torch.empty_like(Ld["q"])
        for n in ("dalpha", "deta", "dtheta", "dgamma"):
            Ld[n] = torch.empty(B, T, H, device=dev)
        Ld["saved"] = torch.empty(lib.atlas_scan_saved_bytes(pp), dtype=torch.uint8, device=dev)
        Ls.append(Ld)
    so = [torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev),
          torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev)]
    di = [torch.empty_like(x) for x in so]

    def one():
        for Ld in Ls:
            L.check(lib.atlas_scan_fwd(pp, P(Ld["q"]), P(Ld["k"]), P(Ld["v"]), P(Ld["alpha"]), P(Ld["eta"]),
                                       P(Ld["theta"]), P(Ld["gamma"]), None, None, None, None, P(Ld["y"]),
                                       *[P(x) for x in so], P(Ld["saved"]), P(ws), nws, sp))
        for Ld in reversed(Ls):
            L.check(lib.atlas_scan_bwd(pp, P(Ld["q"]), P(Ld["k"]), P(Ld["v"]), P(Ld["alpha"]), P(Ld["eta"]),
                                       P(Ld["theta"]), P(Ld["gamma"]), P(Ld["saved"]), P(Ld["dy"]), None, None,
                                       None, None, P(Ld["dq"]), P(Ld["dk"]), P(Ld["dv"]), P(Ld["dalpha"]),
                                       P(Ld["deta"]), P(Ld["dtheta"]), P(Ld["dgamma"]), *[P(x) for x in di],
                                       P(ws), nws, sp))
    one()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(reps):
        one()
    t1.record(stream)
    torch.cuda.synchronize()
    L.check(lib.atlas_scan_status())
    from atlas_b200 import dp
    ms_layer = dp.max_over_ranks(t0.elapsed_time(t1)) / (reps * layers)
    step_ms = ms_layer * c["layers"]
    return {"value": B * T * world / (step_ms / 1e3), "unit": "tokens/s", "dtype": "f32" if f32 else "bf16",
            "pe_ste": bool(pe_ste), "ms_per_layer_fwd_bwd": ms_layer,
            "how": f"{layers} layers fwd+bwd x {reps} timed passes with {'float32' if f32 else 'bf16'} q/k/v/dy, "
                   f"per-layer time x {c['layers']} layers (no all-reduce)"}


def next_rows(dev, stream, peak_tf, hbm):
    """Device-timed figures for the rows beyond the headline scan (rank 0, one GPU):
    the MAG sliding-window attention at config 3's shape (B=2, T=32768, 12 heads x 64,
    window 1024) forward+backward, and the fused layer prologue forward+backward at
    the 170M layer shape (B=8, T=8192, C=768), the Muon Polar Express of the 12 x 4096 x 768
    stack, and config 4's head_dim-128 forward scan (B x H = 96, a 2048-token sample).
    3 untimed + 5 (2 for the scan) timed passes each; every input is larger than L2."""
    import torch
    from atlas_b200.swa import swa_backward, swa_forward
    from atlas_b200.layer_io import LayerGeometry, prologue_backward, prologue_forward
    out = {}
    g = torch.Generator(device=dev)
    g.manual_seed(3)

    def timed(f, n=5):
        for _ in range(3):
            f()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(n):
            f()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / n
    B, T, H, D, W = 2, 32768, 12, 64, 1024
    q, k, v, do = (torch.randn(B, T, H, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
    o, lse = swa_forward(q, k, v, W)
    f_ms = timed(lambda: swa_forward(q, k, v, W))
    b_ms = timed(lambda: swa_backward(q, k, v, o, lse, do, W))
    pairs = B * H * sum(min(t, W) + 1 for t in range(T))  # (query, key) pairs inside the band
    ff, fb = 4 * D * pairs, 10 * D * pairs  # QK^T + PV; QK^T, dO V^T, P^T dO, dS^T Q, dS K
    out["mag_swa"] = {"workload": f"banded RoPE attention B={B} T={T} H={H} D={D} window={W}",
                      "fwd_ms": f_ms, "bwd_ms": b_ms, "fwd_tflops": ff / f_ms / 1e9, "bwd_tflops": fb / b_ms / 1e9,
                      "frac_fwd_bwd": (ff + fb) / ((f_ms + b_ms) / 1e3) / 1e12 / peak_tf,
                      "unit": "TFLOP/s of the band (algorithmic)", "kernels": "swa fwd_kernel, dkv_kernel, dq_kernel"}
    del q, k, v, do, o, lse
    B, T, H, D = 8, 8192, 12, 64
    geo = LayerGeometry(B, T, H, D)
    proj = torch.randn(B * T, geo.proj_stride, device=dev, generator=g).to(torch.bfloat16)
    cw = torch.randn(3, 4, H * D, device=dev, generator=g) * 0.3
    cb = torch.zeros(3, H * D, device=dev)
    poly = torch.ones(2, device=dev)
    gb = torch.zeros(4, H, device=dev)
    qo, ko, vo, gates = prologue_forward(geo, proj, cw, cb, poly, gb)
    pf = timed(lambda: prologue_forward(geo, proj, cw, cb, poly, gb))
    pb = timed(lambda: prologue_backward(geo, proj, cw, cb, poly, gb, qo, ko, vo, gates))
    nb = proj.numel() * 2
    fbytes = nb + 3 * qo.numel() * 2 + 5 * B * T * H * 4        # proj in; q, k, v, 5 gates out
    bbytes = 2 * nb + 3 * qo.numel() * 2 + 5 * B * T * H * 4 + 2 * 3 * qo.numel() * 4  # + dproj out, dc round trip
    out["layer_prologue"] = {"workload": f"prologue B={B} T={T} H={H} D={D} (bf16)", "fwd_ms": pf, "bwd_ms": pb,
                             "fwd_gbs": fbytes / pf / 1e6, "bwd_gbs": bbytes / pb / 1e6,
                             "frac_hbm_fwd": fbytes / pf / 1e6 / hbm, "unit": "GB/s (algorithmic bytes)"}
    del proj, qo, ko, vo, gates
    # Muon orthogonalisation of the 170M model's largest stack (optim.py:68-83)
    from atlas_b200 import ATLAS_PREC_TENSOR, ScanConfig, polar_express, scan_forward
    nb, rows, cols, ns = 12, 4096, 768, 5
    X = torch.randn(nb, rows, cols, device=dev, generator=g)
    pe_ms = timed(lambda: polar_express(X, ns, 0.0, precision=ATLAS_PREC_TENSOR))
    Dm, Em = min(rows, cols), max(rows, cols)
    pe_fl = nb * ns * (4 * Dm * Dm * Em + 2 * Dm ** 3)
    out["muon_pe"] = {"workload": f"Polar Express {ns} steps of {nb} x {rows} x {cols} float32",
                      "ms": pe_ms, "tflops": pe_fl / pe_ms / 1e9, "frac": pe_fl / pe_ms / 1e9 / peak_tf,
                      "unit": "TFLOP/s (algorithmic)", "kernels": "pe_tma gemm_kernel, sumsq, norm_split"}
    del X
    # config 4's head_dim-128 sweep point (B x H = 96), forward only, a 2048-token sample
    B, T, H, D, E = 8, 2048, 12, 128, 512
    nrm = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q, k, v = (nrm(torch.randn(B, T, H, D, device=dev, generator=g)).to(torch.bfloat16) for _ in range(3))
    gate = lambda m: torch.sigmoid(m + 0.5 * torch.randn(B, T, H, device=dev, generator=g))  # noqa: E731
    ga, ge, gt = gate(3.0), gate(-3.0), gate(1.0)
    cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    c4 = timed(lambda: scan_forward(q, k, v, ga, ge, gt, None, None, cfg, need_saved=False), n=2)
    c4_fl = B * T * H * 2 * ns * (4 * D * D * E + 2 * D ** 3)  # Polar Express of W1 and W2 per token-head
    out["config4_d128"] = {"workload": f"forward scan B={B} H={H} T={T} (sample) D={D} E={E} chunk=64 bf16",
                           "ms": c4, "tokens_per_s": B * T / c4 * 1e3, "pe_tflops": c4_fl / c4 / 1e9,
                           "unit": "tokens/s", "kernels": "scan_gen frozen/momentum/memory kernels + pe_cluster Polar Express"}
    del q, k, v, ga, ge, gt
    # config 4's chunk-128 sweep point at head_dim 64 (B x H = 96) on the fused forward
    B, T, H, D = 8, 8192, 12, 64
    q, k, v = (nrm(torch.randn(B, T, H, D, device=dev, generator=g)).to(torch.bfloat16) for _ in range(3))
    ga, ge, gt = gate(3.0), gate(-3.0), gate(1.0)
    cfg = ScanConfig(chunk=128, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    c128 = timed(lambda: scan_forward(q, k, v, ga, ge, gt, None, None, cfg, need_saved=False), n=2)
    out["config4_chunk128"] = {"workload": f"forward scan B={B} H={H} T={T} D={D} E=256 chunk=128 bf16",
                               "ms": c128, "tokens_per_s": B * T / c128 * 1e3,
                               "fwd_tflops": B * T * H * F_FWD(D, 5) / c128 / 1e9,
                               "unit": "tokens/s", "kernels": "tc fwd_kernel (128-token chunks)"}
    del q, k, v, ga, ge, gt
    # config 4's smallest B x H (16 chains), forward only: fewer chains than clusters, so the
    # forward-only call runs the batched forward with the on-chip Polar Express
    B, T, H, D = 1, 8192, 16, 64
    q, k, v = (nrm(torch.randn(B, T, H, D, device=dev, generator=g)).to(torch.bfloat16) for _ in range(3))
    ga, ge, gt = gate(3.0), gate(-3.0), gate(1.0)
    cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    c16 = timed(lambda: scan_forward(q, k, v, ga, ge, gt, None, None, cfg, need_saved=False), n=2)
    out["config4_bh16"] = {"workload": f"forward scan B={B} H={H} T={T} D={D} E=256 chunk=64 bf16 (16 chains)",
                           "ms": c16, "tokens_per_s": B * T / c16 * 1e3,
                           "fwd_tflops": B * T * H * F_FWD(D, 5) / c16 / 1e9,
                           "unit": "tokens/s", "kernels": "scan_gen kernels + pe_cta Polar Express"}
    return out


def gpu_arm(args, rank, world):
    import torch
    from atlas_b200 import _lib as L
    from atlas_b200 import dp
    lib = L.load()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    c = CFG
    B, T, H, D, E, NL = c["B"], c["T"], c["H"], c["D"], c["E"], c["layers"]
    p = L.AtlasScanParams(L.ATLAS_ABI_VERSION, B, T, H, D, E, c["chunk"], c["omega"], c["ns_steps"], 0, 0,
                          L.ATLAS_BF16, L.ATLAS_PREC_TENSOR)
    pp = ctypes.byref(p)
    nsave = lib.atlas_scan_saved_bytes(pp)
    nws = lib.atlas_scan_workspace_bytes(pp)
    if nsave == 0 or nws == 0:
        raise RuntimeError(lib.atlas_last_error_string().decode())
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def unit(x):
        return (x / x.norm(dim=-1, keepdim=True)).bfloat16()
    layers = []
    for _ in range(NL):
        Ld = dict(q=unit(torch.randn(B, T, H, D, device=dev, generator=g)),
                  k=unit(torch.randn(B, T, H, D, device=dev, generator=g)),
                  v=unit(torch.randn(B, T, H, D, device=dev, generator=g)))
        for n, mu in (("alpha", 3.0), ("eta", -3.0), ("theta", 1.0), ("gamma", 0.0)):
            Ld[n] = torch.sigmoid(mu + 0.5 * torch.randn(B, T, H, device=dev, generator=g))
        Ld["dy"] = (torch.randn(B, T, H, D, device=dev, generator=g) * 0.01).bfloat16()
        Ld["y"] = torch.empty_like(Ld["q"])
        Ld["saved"] = torch.empty(nsave, dtype=torch.uint8, device=dev)
        for n in ("dq", "dk", "dv"):
            Ld[n] = torch.empty_like(Ld["q"])
        for n in ("dalpha", "deta", "dtheta", "dgamma"):
            Ld[n] = torch.empty(B, T, H, device=dev)
        layers.append(Ld)
    st_out = [torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev),
              torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev)]
    dst_in = [torch.empty_like(x) for x in st_out]
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    grad_buf = torch.zeros(dp.atlas_param_count(), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    fwd_ev, bwd_ev = [], []

    def fwd(Ld, timed):
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        L.check(lib.atlas_scan_fwd(pp, P(Ld["q"]), P(Ld["k"]), P(Ld["v"]), P(Ld["alpha"]), P(Ld["eta"]),
                                   P(Ld["theta"]), P(Ld["gamma"]), None, None, None, None, P(Ld["y"]),
                                   *[P(x) for x in st_out], P(Ld["saved"]), P(ws), nws, sp))
        if timed:
            e1.record(stream)
            fwd_ev.append((e0, e1))

    def bwd(Ld, timed):
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        L.check(lib.atlas_scan_bwd(pp, P(Ld["q"]), P(Ld["k"]), P(Ld["v"]), P(Ld["alpha"]), P(Ld["eta"]),
                                   P(Ld["theta"]), P(Ld["gamma"]), P(Ld["saved"]), P(Ld["dy"]), None, None,
                                   None, None, P(Ld["dq"]), P(Ld["dk"]), P(Ld["dv"]), P(Ld["dalpha"]),
                                   P(Ld["deta"]), P(Ld["dtheta"]), P(Ld["dgamma"]), *[P(x) for x in dst_in],
                                   P(ws), nws, sp))
        if timed:
            e1.record(stream)
            bwd_ev.append((e0, e1))

    copy_stream = torch.cuda.Stream(dev)

    def step(timed=False, host=None):
        # End-to-end steps move every layer's inputs host -> device and its gradients
        # device -> host on a copy stream, overlapped with the scan kernels; the step
        # ends only when the last gradient has reached the host.
        if host is not None:
            copy_stream.wait_stream(stream)  # the previous step is done with the buffers
            ready = []
            with torch.cuda.stream(copy_stream):
                for Ld in layers:
                    for n in ("q", "k", "v", "alpha", "eta", "theta", "gamma", "dy"):
                        Ld[n].copy_(host[n], non_blocking=True)
                    ready.append(copy_stream.record_event())
        for i, Ld in enumerate(layers):
            if host is not None:
                stream.wait_event(ready[i])
            fwd(Ld, timed)
        for Ld in reversed(layers):
            bwd(Ld, timed)
            if host is not None:
                copy_stream.wait_stream(stream)
                with torch.cuda.stream(copy_stream):
                    for n in ("dq", "dk", "dv", "dalpha", "deta", "dtheta", "dgamma"):
                        host["out_" + n].copy_(Ld[n], non_blocking=True)
        dp.allreduce_mean_(grad_buf)
        if host is not None:
            stream.wait_stream(copy_stream)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    L.check(lib.atlas_scan_status())
    clocks = Clocks(os.path.join(tempfile.gettempdir(), f"atlas_bench_clocks_{os.getpid()}_rank{rank}.csv"))
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step(timed=True)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ck = clocks.stop(dev.index)
    L.check(lib.atlas_scan_status())
    ms = dp.max_over_ranks(t0.elapsed_time(t1)) / args.steps
    tokens = B * T * world
    value = tokens / (ms / 1e3)
    fwd_ms = sum(a.elapsed_time(b) for a, b in fwd_ev) / len(fwd_ev)
    bwd_ms = sum(a.elapsed_time(b) for a, b in bwd_ev) / len(bwd_ev)

    # ---- end to end: host inputs in, host gradients out, every step ----
    host = {n: torch.empty_like(layers[0][n], device="cpu").pin_memory().copy_(layers[0][n])
            for n in ("q", "k", "v", "alpha", "eta", "theta", "gamma", "dy")}
    for n in ("dq", "dk", "dv", "dalpha", "deta", "dtheta", "dgamma"):
        host["out_" + n] = torch.empty_like(layers[0][n], device="cpu").pin_memory()
    h2d = NL * sum(host[n].numel() * host[n].element_size()
                   for n in ("q", "k", "v", "alpha", "eta", "theta", "gamma", "dy"))
    d2h = NL * sum(host["out_" + n].numel() * host["out_" + n].element_size()
                   for n in ("dq", "dk", "dv", "dalpha", "deta", "dtheta", "dgamma"))
    e2e_steps = max(1, min(args.steps, 2))
    e2e = None
    if not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(e2e_steps):
            step(host=host)
        t1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = dp.max_over_ranks(t0.elapsed_time(t1)) / e2e_steps
        e2e = tokens / (e2e_ms / 1e3)

    f32 = None if args.no_f32 else f32_mode(lib, L, dev, stream, sp, p, nws, ws, g, world)
    ste = None if args.no_f32 else f32_mode(lib, L, dev, stream, sp, p, nws, ws, g, world, f32=False, pe_ste=1)
    peak_tf, hbm, peak_kind = _peaks()
    f_bwd = B * T * H * F_BWD(D, c["ns_steps"])
    f_fwd = B * T * H * F_FWD(D, c["ns_steps"])
    dom_ms, dom_f, dom = (bwd_ms, f_bwd, "tc_bwd_kernel") if bwd_ms >= fwd_ms else (fwd_ms, f_fwd, "tc_fwd_kernel")
    achieved = dom_f / (dom_ms / 1e3) / 1e12
    out = {
        "metric": METRIC, "value": value, "value_per_gpu": value / world, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"170M Atlas scan fwd+bwd, {NL} layers, per GPU B={B} T={T} H={H} D={D} "
                               f"E={E} chunk=64 omega=16 ns=5 pe_ste=False", "model": "atlas-170M (scan only)",
                   "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world}",
                   "l2": "inputs larger than L2 (per-layer inputs ~420 MB)",
                   "grad_allreduce_params": grad_buf.numel()},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak_tf,
                     "unit": "TFLOP/s", "frac": achieved / peak_tf,
                     "traffic": NCU_TRAFFIC[dom] * (B * T * H) / NCU_TOKEN_HEADS,
                     "traffic_unit": "bytes per launch",
                     "traffic_source": "ncu capture at T=256 scaled by token-heads",
                     "peak_source": f"bf16_tflops_sustained ({peak_kind})",
                     "fwd_ms_per_layer": fwd_ms, "bwd_ms_per_layer": bwd_ms},
        "gpu_launches": 2 * NL * args.steps,
        "clocks": ck,
        "f32_activations": f32,
        "pe_ste": ste,
    }
    if rank == 0 and world == 1 and not args.no_next:
        out["next_rows"] = next_rows(dev, stream, peak_tf, hbm)
    if rank == 0 and world == 1 and not args.no_cpu:
        v, dt, cores = cpu_baseline()
        out["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                               "sample": f"{CPU_SAMPLE_TEXT} ({dt:.1f} s)"}
    if rank == 0:
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--layers", type=int, default=CFG["layers"], help="profiling only: fewer layers")
    ap.add_argument("--seq", type=int, default=CFG["T"], help="profiling only: shorter sequences")
    ap.add_argument("--no-e2e", action="store_true", help="profiling only: skip the end-to-end leg")
    ap.add_argument("--no-f32", action="store_true", help="skip the float32-activation and pe_ste legs")
    ap.add_argument("--no-next", action="store_true", help="skip the attention / prologue leg")
    args = ap.parse_args()
    if args.layers != CFG["layers"] or args.seq != CFG["T"]:
        CFG["layers"], CFG["T"] = args.layers, args.seq
        args.no_cpu = True
        args.no_f32 = True
        args.no_next = True
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if world > 1:
        from atlas_b200 import dp
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dp.init("nccl")
    gpu_arm(args, rank, world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
