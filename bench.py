"""Benchmark of the compressed-KV decode hot path (sd1 1-bit codec) on B200.

Workload: Llama-3-8B attention shapes — 32 layers,
32 query / 8 KV heads, head_dim 128 — batch 1 at 32768-token context: the last
512 tokens sit in the fp16 window, the other 32256 are encoded (DCT, tiles of
64) into the 1-bit store; each decode step selects the top 16 tiles per KV
head and attends window + selected tiles, layer after layer.  Synthetic data
of the config-0 distribution stands in for a random-init model's K/V and
queries (there is no checkpoint or dataset here).

A "step" = one decode step of all 32 layers (2 kernels per layer).  The 32
layers' stores and windows (~395 MB) exceed L2 (126 MB), so every step reads
its inputs from HBM.  With --gpus N (torchrun) the KV heads are sharded: each
rank holds Hkv/N heads of a batch of N sequences (weak scaling, no
collective); value counts sequence-steps of the whole job.

--impl reference times the reference algorithm's CPU path (the int4w
retrieve_topk token branch + window/retrieved softmax, restated in
oracle/int4w_ref_cpu.py) on the host cores at the same shapes.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rina-1bit-kv_b200"))
sys.path.insert(0, ROOT)

LAYERS, HQ, HKV, D = 32, 32, 8, 128
CTX, WIN, TILE, KSEL, KIND = 32768, 512, 64, 16, "dct"
T_STORED = CTX - WIN                      # 32256
NT = T_STORED // TILE                     # 504
METRIC = "decode-attn steps/s + achieved HBM GB/s at 32k ctx; KV encode tokens/s"


def step_bytes_per_layer(hkv, batch):
    """Algorithmic bytes of one layer-step (sd1): scan all K bits + K scales,
    re-read the selected K tiles, selected V bits + scales, window K and V in
    fp16, q in and out in bf16."""
    kb, sc = TILE * D // 8, 2 * D
    select = batch * hkv * NT * (kb + sc)
    attend = batch * hkv * (KSEL * 2 * (kb + sc) + WIN * D * 2 * 2) + 2 * batch * hkv * (HQ // HKV) * D * 2
    return select, attend


def clocks_sampler():
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        return subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"],
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def clocks_summary(proc, dev_index):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9 or f[0] != str(dev_index):
            continue
        try:
            sm.append(float(f[1]))
            mx = float(f[2])
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ----------------------------------------------------------------- GPU arm --

# batched decode stress, batch 32 x 16384 context, window
# 256, top 16 tiles of 64 (Llama-3-8B attention shapes, 32 q / 8 KV heads).
B2, CTX2, WIN2, L2_LAYERS = 32, 16384, 256, 4
NT2 = (CTX2 - WIN2) // TILE  # 252


def run_batched(dev, g, peak):
    """Secondary measurement on configs[2] at one GPU: the decode step of a
    layer over a batch of 32 sequences, timed as a CUDA graph over 4 layers
    (4 x 127 MB of stores + windows, larger than L2), then the select and
    attend kernels alone.  Bytes are the algorithmic bytes of the step: the
    select reads every stored tile's K bits + K scales, the attention the
    selected tiles' K/V bits and scales, the fp16 window rows, q and out."""
    import torch

    from kvr_b200 import kernels as K
    from kvr_b200 import _native as N

    stores, wins = [], []
    for li in range(L2_LAYERS):
        scale = torch.exp(torch.randn(HKV, D, device=dev, generator=g))
        idx = torch.randint(0, D, (HKV, 4), device=dev, generator=g)
        scale.scatter_(1, idx, scale.gather(1, idx) * 20)
        k = (torch.randn(B2, NT2 * TILE, HKV, D, device=dev, generator=g) * scale).to(torch.bfloat16)
        v = torch.randn(B2, NT2 * TILE, HKV, D, device=dev, generator=g).to(torch.bfloat16)
        st = K.Sd1Store(B2, HKV, NT2, TILE, KIND, dev)
        K.sd1_encode(st, k, v)
        stores.append(st)
        del k, v
        wins.append((torch.randn(B2, WIN2, HKV, D, device=dev, generator=g).half(),
                     torch.randn(B2, WIN2, HKV, D, device=dev, generator=g).half()))
    q = torch.randn(L2_LAYERS, B2, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    ws = torch.zeros(N.call("kvr_sd1_workspace_bytes", B2, HQ, HKV, NT2, TILE, KSEL, WIN2, 0) + 256,
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def timed(fn, reps=30):
        with torch.cuda.stream(stream):
            fn()
            fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                gr.replay()
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps / L2_LAYERS

    def step():
        for li in range(L2_LAYERS):
            wk, wv = wins[li]
            K.sd1_decode_step(stores[li], q[li], KSEL, wk, wv, WIN2, out=out[li], ws=ws)

    ms_step = timed(step)
    sels = [K.sd1_select(stores[li], q[li], KSEL) for li in range(L2_LAYERS)]

    def sel_only():
        for li in range(L2_LAYERS):
            K.sd1_select(stores[li], q[li], KSEL)

    def att_only():
        for li in range(L2_LAYERS):
            s_, _, qp = sels[li]
            wk, wv = wins[li]
            K.sd1_attend(stores[li], q[li], qp, s_, wk, wv, WIN2, out_dtype=torch.bfloat16)

    ms_sel, ms_att = timed(sel_only), timed(att_only)
    kb, sc = TILE * D // 8, D * 2
    sel_b = B2 * HKV * NT2 * (kb + sc)
    att_b = B2 * HKV * (KSEL * 2 * (kb + sc) + WIN2 * D * 2 * 2) + 2 * B2 * HQ * D * 2
    gbs = (sel_b + att_b) / (ms_step / 1e3) / 1e9
    res = {"workload": "configs[2] batched decode stress: batch 32 x 16384 context, window 256, "
                       "top 16 tiles of 64, dct, Llama-3-8B attention shapes",
           "layers_in_graph": L2_LAYERS, "us_per_layer": round(ms_step * 1e3, 2),
           "sequence_layer_steps_per_s": round(B2 / (ms_step / 1e3), 1),
           "bytes_per_layer": sel_b + att_b, "hbm_gbs": round(gbs, 1), "peak": peak,
           "frac": round(gbs / peak, 4), "select_us": round(ms_sel * 1e3, 2), "attend_us": round(ms_att * 1e3, 2),
           "select_bytes": sel_b, "attend_bytes": att_b,
           "select_gbs": round(sel_b / (ms_sel / 1e3) / 1e9, 1), "attend_gbs": round(att_b / (ms_att / 1e3) / 1e9, 1),
           "kernels": "sd1_score_flat_kernel (popcount tile scores over equal (row, tile) ranges + top-k, "
                      "streams the window into L2) -> "
                      "attn_rows_kernel (mma.sync pieces)"}
    del stores, wins, sels
    torch.cuda.empty_cache()
    return res


def run_gpu(args, rank, world, local_rank):
    import torch

    from kvr_b200 import kernels as K
    from kvr_b200 import _native as N

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hkv = HKV // world            # heads owned by this rank
    hq = HQ // world
    B = world                     # sequences in the job (weak scaling)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def cfg0_kv(n):
        scale = torch.exp(torch.randn(hkv, D, device=dev, generator=g))
        idx = torch.randint(0, D, (hkv, 4), device=dev, generator=g)
        scale.scatter_(1, idx, scale.gather(1, idx) * 20)
        k = (torch.randn(B, n, hkv, D, device=dev, generator=g) * scale).to(torch.bfloat16)
        v = torch.randn(B, n, hkv, D, device=dev, generator=g).to(torch.bfloat16)
        return k, v

    # ---- prefill encode of every layer (also the encode measurement)
    stores, wins = [], []
    enc_ms = []
    st_ev, en_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for li in range(LAYERS):
        k, v = cfg0_kv(CTX)
        st = K.Sd1Store(B, hkv, NT, TILE, KIND, dev)
        reps = 3 if li == 0 else 1
        for r in range(reps):
            st.n_tiles = 0
            torch.cuda._sleep(100000)  # the GPU is busy while the host enqueues: events bracket the kernel
            st_ev.record()
            K.sd1_encode(st, k[:, :T_STORED], v[:, :T_STORED])
            en_ev.record()
            torch.cuda.synchronize()
            if li > 0 or r > 0:
                enc_ms.append(st_ev.elapsed_time(en_ev))
        stores.append(st)
        wins.append((k[:, T_STORED:].to(torch.float16).contiguous(), v[:, T_STORED:].to(torch.float16).contiguous()))
        del k, v
    enc_s = statistics.median(enc_ms) / 1e3
    enc_tok_layer = B * T_STORED / enc_s
    enc_bytes = B * T_STORED * hkv * (2 * D * 2 + 2 * D // 8) + B * hkv * NT * 2 * 2 * D

    # ---- decode step: all layers, q per layer
    qs = torch.randn(LAYERS, B, hq, D, device=dev, generator=g).to(torch.bfloat16)
    outs = torch.empty_like(qs)
    need = N.call("kvr_sd1_workspace_bytes", B, hq, hkv, NT, TILE, KSEL, WIN, 0)
    ws = torch.zeros(need + 256, dtype=torch.uint8, device=dev)

    def step(q_all, o_all):
        for li in range(LAYERS):
            wk, wv = wins[li]
            K.sd1_decode_step(stores[li], q_all[li], KSEL, wk, wv, WIN, out=o_all[li], ws=ws)

    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    graph, mode = None, "eager"
    with torch.cuda.stream(stream):
        for _ in range(2):
            step(qs, outs)
    torch.cuda.synchronize()
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
                step(qs, outs)
            mode = "cuda_graph"
        except Exception as e:  # noqa: BLE001 - report and fall back to eager launches
            print(f"[bench] graph capture failed, eager launches: {e}", file=sys.stderr)
            graph = None
            torch.cuda.synchronize()

    def run_once():
        if graph is not None:
            graph.replay()
        else:
            step(qs, outs)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run_once()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clk = clocks_sampler() if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            run_once()
        e1.record(stream)
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([t_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
        dist.barrier()
    clocks = clocks_summary(clk, local_rank) if rank == 0 else None
    ms_per_step = t_ms / args.steps

    # ---- per-kernel durations (eager, events on the launching stream)
    sel_b, att_b = step_bytes_per_layer(hkv, B)
    qp = torch.empty(B, hq, D, dtype=torch.float32, device=dev)
    sel = torch.empty(B, hkv, KSEL, dtype=torch.int32, device=dev)
    sws = torch.zeros(N.call("kvr_sd1_select_workspace_bytes", B, hkv, NT) + 256, dtype=torch.uint8, device=dev)
    aws = torch.zeros(N.call("kvr_sd1_attend_workspace_bytes", B, hq, hkv, TILE, KSEL, WIN, 0) + 256,
                      dtype=torch.uint8, device=dev)
    # each timed launch sits behind a GPU sleep, so the host-side enqueue cost
    # of the eager call is hidden and the events bracket only the kernel
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    t_sel, t_att = [], []
    P = N.ptr
    with torch.cuda.stream(stream):
        sp = stream.cuda_stream
        for rep in range(3):
            for li in range(LAYERS):
                st = stores[li]
                wk, wv = wins[li]
                torch.cuda._sleep(200000)
                ev[0].record(stream)
                N.call("kvr_sd1_select", P(qs[li]), N.dtype_code(qs[li]), B, hq, hkv, P(st.kbits), P(st.kscale),
                       st.nt_cap, st.n_tiles, TILE, N.TRANSFORMS[KIND], KSEL, 0, 0, 0, P(sel), None, P(qp), P(sws),
                       sws.numel(), sp)
                ev[1].record(stream)
                torch.cuda._sleep(200000)
                ev[2].record(stream)
                N.call("kvr_sd1_attend", P(qs[li]), N.dtype_code(qs[li]), P(qp), B, hq, hkv, P(wk), P(wv), WIN, WIN,
                       None, None, 0, P(st.kbits), P(st.kscale), P(st.vbits), P(st.vscale), st.nt_cap, TILE,
                       N.TRANSFORMS[KIND], P(sel), KSEL, 0.0, P(outs[li]), N.dtype_code(outs[li]), None, P(aws),
                       aws.numel(), sp)
                ev[3].record(stream)
                ev[3].synchronize()
                if rep:
                    t_sel.append(ev[0].elapsed_time(ev[1]))
                    t_att.append(ev[2].elapsed_time(ev[3]))
    ms_sel, ms_att = statistics.mean(t_sel), statistics.mean(t_att)

    # ---- end to end through the public API with pinned host buffers
    q_host = qs.cpu().pin_memory()
    o_host = torch.empty(outs.shape, dtype=outs.dtype).pin_memory()
    q_dev = torch.empty_like(qs)
    e2e_steps = max(3, min(args.steps, 100))
    with torch.cuda.stream(stream):
        for i in range(e2e_steps + 2):
            if i == 2:
                e0.record(stream)
            q_dev.copy_(q_host, non_blocking=True)
            for li in range(LAYERS):
                wk, wv = wins[li]
                K.sd1_decode_step(stores[li], q_dev[li], KSEL, wk, wv, WIN, out=outs[li], ws=ws)
            o_host.copy_(outs, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())

    # ---- tcgen05 prefill tile scoring (secondary line): a 4096-query chunk
    # of prefill positions scored against layer 0's store (batch-1 stores only)
    prefill = None
    if B == 1:
        nq_pf = 4096
        q_pf = torch.randn(nq_pf, hq, D, device=dev, generator=g).to(torch.bfloat16)
        for _ in range(3):
            K.sd1_prefill_scores(stores[0], q_pf)
        torch.cuda.synchronize()
        reps = 20
        e0.record()
        for _ in range(reps):
            K.sd1_prefill_scores(stores[0], q_pf)
        e1.record()
        torch.cuda.synchronize()
        pf_ms = e0.elapsed_time(e1) / reps
        pf_flops = 2.0 * nq_pf * hkv * stores[0].n_tiles * TILE * D
        pf_peak = None
        try:
            pf_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
            pf_src = "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
        except (OSError, KeyError, ValueError):
            pf_peak, pf_src = 1590.0, "fallback"
        pf_tf = pf_flops / (pf_ms / 1e3) / 1e12
        prefill = {"kernel": "prefill_scores_kernel (tcgen05.mma kind::f16) + q prep", "queries": nq_pf,
                   "tokens": stores[0].n_tiles * TILE, "kv_heads": hkv, "ms_per_launch": round(pf_ms, 5),
                   "flops_per_launch": pf_flops, "achieved": round(pf_tf, 1), "unit": "TFLOP/s",
                   "peak": pf_peak, "frac": round(pf_tf / pf_peak, 4), "peak_source": pf_src,
                   "bound": "tensor"}
        del q_pf

    peak, peak_kind = measured_peak_hbm()
    batched = None
    if world == 1 and not args.no_batched:
        batched = run_batched(dev, g, peak)
    traffic = None
    try:  # DRAM bytes per launch from the committed ncu capture of this workload
        tj = json.load(open(os.path.join(ROOT, "profiles", "traffic_config1.json")))["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        tj = {}
    layer_bytes = sel_b + att_b
    dom = "select" if ms_sel >= ms_att else "attend"
    dom_bytes, dom_ms = (sel_b, ms_sel) if dom == "select" else (att_b, ms_att)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    if world == 1:
        traffic = tj.get("sd1_score_kernel" if dom == "select" else "attn_kernel")
    res = {
        "metric": METRIC,
        "value": round(B * 1e3 / ms_per_step, 3),
        "unit": "sequence decode-steps/s (32 layers per step)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 q / fp16 window / 1-bit sd1 codes, fp32 accumulate",
        "data": "synthetic: config-0 K/V distribution (log-normal channel scales, 4 outlier channels x20), N(0,1) q",
        "config": {"workload": "configs[1] Llama-3-8B attention shapes, decode over sd1 store",
                   "layers": LAYERS, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context": CTX,
                   "window": WIN, "tile": TILE, "top_k_tiles": KSEL, "transform": KIND,
                   "batch_per_rank": B, "kv_heads_per_rank": hkv, "parallelism": f"kv-head shard x{world}",
                   "l2": "inputs larger than L2 (~395 MB of stores+windows per step)", "launch": mode},
        "hbm_gbs": round(LAYERS * layer_bytes * world / (ms_per_step / 1e3) / 1e9, 1),
        "encode": {"layer_tokens_per_s": round(enc_tok_layer * world, 1),
                   "prefill_tokens_per_s": round(enc_tok_layer * world / LAYERS, 1),
                   "hbm_gbs": round(enc_bytes / enc_s / 1e9, 1), "ms_per_layer": round(enc_s * 1e3, 4),
                   "tokens_per_layer": B * T_STORED},
        "roofline": {"bound": "hbm", "kernel": f"sd1_{dom}", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic, "traffic_source": "profiles/traffic_config1.json (ncu)",
                     "algorithmic_bytes_per_launch": dom_bytes, "ms_per_launch": round(dom_ms, 5),
                     "select_ms": round(ms_sel, 5), "attend_ms": round(ms_att, 5),
                     "select_bytes": sel_b, "attend_bytes": att_b},
        "e2e": {"value": round(B * 1e3 / e2e_ms, 3), "unit": "sequence decode-steps/s (32 layers per step)",
                "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
                "d2h_bytes_per_step": o_host.numel() * o_host.element_size(), "path": "kvr_b200.kernels eager API"},
        "prefill_scores": prefill,
        "batched": batched,
        "gpu_launches": args.steps * LAYERS * 2,
        "clocks": clocks,
    }
    return res


# --------------------------------------------------------------- CPU arm --

def cpu_reference(sample_layers, threads=None):
    """The reference algorithm's CPU decode path on the host cores, timed per
    layer on a bounded sample and scaled to a 32-layer step."""
    import torch

    from oracle import int4w_ref_cpu as C

    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    case = C.make_case(seed=0, n_stored=T_STORED, window=WIN, n_kv=HKV, n_q=HQ, d=D)
    top_k = KSEL * TILE
    C.decode_layer(case, top_k)  # warm-up
    ts = []
    for i in range(sample_layers):
        t0 = time.perf_counter()
        C.decode_layer(case, top_k, q_index=i)
        ts.append(time.perf_counter() - t0)
    layer_s = statistics.median(ts)
    step_s = layer_s * LAYERS
    return {"value": round(1.0 / step_s, 5), "unit": "sequence decode-steps/s (32 layers per step)",
            "cores": threads, "kind": "port",
            "sample": f"{sample_layers} single-layer decode steps (int4w retrieve_topk token branch, top_k={top_k}, "
                      f"{T_STORED} stored + {WIN} window tokens, 8 KV / 32 Q heads), median x {LAYERS} layers",
            "layer_ms": round(layer_s * 1e3, 3)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the configs[2] batched measurement")
    ap.add_argument("--batched-only", action="store_true",
                    help="run only the configs[2] batched measurement (one GPU; for profiling)")
    ap.add_argument("--cpu-sample", type=int, default=8, help="layers timed for the CPU baseline")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    # stdout carries exactly one JSON line: anything else written to file
    # descriptor 1 (library banners, warnings) is sent to stderr, and the
    # result goes to a private copy of the original stdout
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    def emit(obj):
        os.write(json_fd, (json.dumps(obj) + "\n").encode())

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_reference(max(args.steps, 3))
        line = {"metric": METRIC, "value": cb["value"], "unit": cb["unit"], "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / cb["value"], 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (reference CPU path)",
                "data": "synthetic: config-0 K/V distribution", "impl": "reference",
                "config": {"workload": "configs[1] Llama-3-8B attention shapes, int4w reference decode path",
                           "layers": LAYERS, "context": CTX, "window": WIN, "top_k_tokens": KSEL * TILE},
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        emit(line)
        return

    if args.batched_only:
        import torch
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(1234)
        emit({"batched": run_batched(dev, g, measured_peak_hbm()[0])})
        return

    if world > 1:
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    res = run_gpu(args, rank, world, local_rank)
    if rank == 0:
        if world == 1:
            res["cpu_baseline"] = cpu_reference(args.cpu_sample)
        emit(res)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
