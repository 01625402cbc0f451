"""Phase breakdown of one batch-1 sd1 decode layer (BASELINE configs[1]
shapes: 8 KV / 32 query heads, 32256 stored tokens in tiles of 64, window
512, top 16 tiles, DCT), from %globaltimer stamps compiled into a separate
trace build of the library (KVR_TRACE_POINT; python -m kvr_b200._build
--trace).  The product library carries no stamps.

    python rina-1bit-kv_b200/phase_trace.py [--layers 32] [--reps 30]
    python rina-1bit-kv_b200/phase_trace.py --batched   # configs[2] flat tile scan
    python rina-1bit-kv_b200/phase_trace.py --split     # the two-kernel batch-1 step

A 32-layer step is captured in a CUDA graph as in bench.py and replayed;
after each replay the stamps of the last layer's two kernels are read back
(every launch overwrites the same slots) and expressed in microseconds from
the first stamp of that layer's selection kernel.  Prints a markdown table of
the medians over the replays.  Stamps are taken by thread 0 of each CTA;
"first"/"last" are the minimum / maximum over the CTAs of a group.
"""
import argparse
import ctypes
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TRACE_LIB = os.path.join(HERE, "kvr_b200", "lib", "libkvr_b200_trace.so")
os.environ["KVR_B200_LIB"] = TRACE_LIB
sys.path.insert(0, HERE)

import torch  # noqa: E402

from kvr_b200 import _native as N  # noqa: E402
from kvr_b200 import kernels as K  # noqa: E402

D, HQ, HKV, CTX, WIN, TILE, KSEL = 128, 32, 8, 32768, 512, 64, 16
NT = (CTX - WIN) // TILE
SLOTS = 2048  # trace slots per kernel id


def read(fn):
    buf = (ctypes.c_ulonglong * (4 * SLOTS * 8))()
    rc = fn(buf, 4 * SLOTS * 8)
    if rc != 0:
        raise RuntimeError("trace readback failed")
    return buf


def stamps(buf, kernel, blocks, point):
    out = []
    for b in blocks:
        v = buf[(kernel * SLOTS + b) * 8 + point]
        if v:
            out.append(v)
    return out


def batched_scan(reps):
    """Phases of sd1_score_flat_kernel (trace kernel id 2) at configs[2]
    shapes: 32 sequences x 8 KV heads x 252 tiles of 64 (16384 context less a
    256 window), top 16, DCT, bf16 q.  Each replay is one standalone
    selection call after a 256 MiB memset (cold L2); stamps are per CTA."""
    B, NT2 = 32, 252
    lib = N.lib()
    rd = lib.kvr_debug_trace_sd1
    rd.argtypes = [ctypes.c_void_p, ctypes.c_int]
    rd.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    scale = torch.exp(torch.randn(HKV, D, device=dev, generator=g))
    k = (torch.randn(B, NT2 * TILE, HKV, D, device=dev, generator=g) * scale).to(torch.bfloat16)
    v = torch.randn(B, NT2 * TILE, HKV, D, device=dev, generator=g).to(torch.bfloat16)
    st = K.Sd1Store(B, HKV, NT2, TILE, "dct", dev)
    K.sd1_encode(st, k, v)
    del k, v
    q = torch.randn(B, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rows = {}
    for _ in range(reps):
        flush.zero_()
        K.sd1_select(st, q, KSEL)
        torch.cuda.synchronize()
        buf = read(rd)
        T = lambda b, p: buf[(2 * SLOTS + b) * 8 + p]  # noqa: E731
        blocks = [b for b in range(SLOTS) if T(b, 0)]
        t0 = min(T(b, 0) for b in blocks)
        V = lambda b, p: T(b, p) if T(b, p) >= t0 else 0  # noqa: E731  (older launches' stamps)
        med = lambda xs: statistics.median(list(xs)) / 1e3  # noqa: E731

        def add(name, val):
            rows.setdefault(name, []).append(val)

        add("CTAs", len(blocks))
        add("start -> copy ring issued (median CTA)", med(T(b, 6) - T(b, 0) for b in blocks))
        add("grid dependency wait (median CTA)", med(T(b, 7) - T(b, 6) for b in blocks))
        add("q' of the CTA's rows formed (median CTA)", med(T(b, 1) - T(b, 7) for b in blocks))
        add("tile scan (median CTA)", med(T(b, 2) - T(b, 1) for b in blocks))
        add("tile scan (slowest CTA)", max(T(b, 2) - T(b, 1) for b in blocks) / 1e3)
        sel = [max(V(b, 4), V(b, 5)) - T(b, 2) for b in blocks if max(V(b, 4), V(b, 5))]
        add("row selection by the completing CTA (median)", med(sel))
        add("row selection (slowest)", max(sel) / 1e3)
        add("last CTA done (from first start)",
            max(max(V(b, 3), V(b, 4), V(b, 5)) for b in blocks) / 1e3 - t0 / 1e3)
    # the batched attention kernel (attn_rows_kernel, trace kernel id 1) on
    # the selection above: window of 256 fp16 rows + 16 tiles per row
    WIN2 = 256
    wk = torch.randn(B, WIN2, HKV, D, device=dev, generator=g).half()
    wv = torch.randn(B, WIN2, HKV, D, device=dev, generator=g).half()
    rd_att = lib.kvr_debug_trace_attn
    rd_att.argtypes = [ctypes.c_void_p, ctypes.c_int]
    rd_att.restype = ctypes.c_int
    sel, _, qp = K.sd1_select(st, q, KSEL)
    for _ in range(reps):
        flush.zero_()
        K.sd1_attend(st, q, qp, sel, wk, wv, WIN2, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        buf = read(rd_att)
        T = lambda b, p: buf[(1 * SLOTS + b) * 8 + p]  # noqa: E731
        blocks = [b for b in range(SLOTS) if T(b, 0) and T(b, 6) >= T(b, 0)]
        t0 = min(T(b, 0) for b in blocks)
        med = lambda xs: statistics.median(list(xs)) / 1e3  # noqa: E731

        def add(name, val):
            rows.setdefault(name, []).append(val)

        add("attend: CTAs", len(blocks))
        add("attend: last CTA start", max(T(b, 0) for b in blocks) / 1e3 - t0 / 1e3)
        add("attend: q staged as B fragments (median CTA)", med(T(b, 1) - T(b, 0) for b in blocks))
        add("attend: 32-token pieces, all warps (median CTA)", med(T(b, 2) - T(b, 1) for b in blocks))
        add("attend: pieces (slowest CTA)", max(T(b, 2) - T(b, 1) for b in blocks) / 1e3)
        add("attend: fold of the 8 warp states (median CTA)", med(T(b, 3) - T(b, 2) for b in blocks))
        add("attend: finish, inverse transform + output (median CTA)", med(T(b, 6) - T(b, 3) for b in blocks))
        add("attend: last CTA done (from first start)", max(T(b, 6) for b in blocks) / 1e3 - t0 / 1e3)
    print("| phase (configs[2] flat tile scan) | us (median over replays) |")
    print("|---|---|")
    for name, vals in rows.items():
        val = statistics.median(vals)
        print(f"| {name} | {val:.0f} |" if name.endswith("CTAs") else f"| {name} | {val:.2f} |")


def cluster_phases(lib, gr, stream, reps, layer_us, layers):
    """Phases of the one-kernel step (sd1_dsmem_step_kernel, trace kernel id 0
    of its translation unit): one cluster of C CTAs per KV head; times are
    from the first CTA start of the last layer."""
    rd = lib.kvr_debug_trace_dsmem
    rd.argtypes = [ctypes.c_void_p, ctypes.c_int]
    rd.restype = ctypes.c_int
    rows = {}
    names = {1: "grid dependency wait passed", 2: "q' formed", 3: "store staged + tile scan done",
             4: "list built + cluster barrier 1", 5: "lists exchanged + rank selection done",
             6: "tiles attended, warp states ready", 7: "rows pushed + cluster barrier 2"}
    names1 = {0: "  store staged (scan may start)", 1: "  selection done, tile copies issued (warps 0-3)",
              2: "  exact rows attended (warps 4-7)", 3: "  selected tiles landed",
              4: "  selected tiles attended (warp 0)", 5: "  merge: weights formed (merging CTAs)",
              6: "  merge: rows combined", 7: "  merge: inverse transform + output written"}
    for _ in range(reps):
        with torch.cuda.stream(stream):
            gr.replay()
        torch.cuda.synchronize()
        buf = read(rd)
        blocks = [b for b in range(SLOTS) if buf[b * 8]]
        t0 = min(stamps(buf, 0, blocks, 0))
        us = lambda x: (x - t0) / 1e3  # noqa: E731

        def add(name, v):
            rows.setdefault(name, []).append(v)

        add("CTAs", len(blocks))
        sms = [buf[(2 * SLOTS + b) * 8] for b in blocks]
        add("distinct SMs", len(set(sms)))
        add("first CTA starts", 0.0)
        add("last CTA starts", us(max(stamps(buf, 0, blocks, 0))))
        for p, name in names.items():
            v = stamps(buf, 0, blocks, p)
            add(f"{name} (first CTA)", us(min(v)))
            add(f"{name} (last CTA)", us(max(v)))
        for p, name in names1.items():
            v = [x for x in stamps(buf, 1, blocks, p) if x >= t0]
            if v:
                add(f"{name} (first CTA)", us(min(v)))
                add(f"{name} (last CTA)", us(max(v)))
    print(f"graph-replayed step: {layer_us:.2f} us per layer ({layers} layers)\n")
    print("| phase (last layer of the step, one-kernel cluster step) | us from the layer's first CTA start (median) |")
    print("|---|---|")
    for name, vals in rows.items():
        val = statistics.median(vals)
        print(f"| {name} | {val:.0f} |" if name in ("CTAs", "distinct SMs") else f"| {name} | {val:.2f} |")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--batched", action="store_true", help="configs[2] flat tile scan phases instead")
    ap.add_argument("--split", action="store_true", help="the two-kernel step (select + attend) instead of "
                    "the one-kernel cluster step")
    args = ap.parse_args()
    if not os.path.exists(TRACE_LIB):
        raise SystemExit(f"{TRACE_LIB} missing: python -m kvr_b200._build --trace (from rina-1bit-kv_b200/)")
    if args.batched:
        batched_scan(args.reps)
        return
    lib = N.lib()
    if args.split:
        lib.kvr_set_sd1_step_path(1)
    rd_sel = lib.kvr_debug_trace_sd1
    rd_att = lib.kvr_debug_trace_attn
    for f in (rd_sel, rd_att):
        f.argtypes = [ctypes.c_void_p, ctypes.c_int]
        f.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    stores, wins = [], []
    for _ in range(args.layers):
        scale = torch.exp(torch.randn(HKV, D, device=dev, generator=g))
        k = (torch.randn(1, NT * TILE, HKV, D, device=dev, generator=g) * scale).to(torch.bfloat16)
        v = torch.randn(1, NT * TILE, HKV, D, device=dev, generator=g).to(torch.bfloat16)
        st = K.Sd1Store(1, HKV, NT, TILE, "dct", dev)
        K.sd1_encode(st, k, v)
        stores.append(st)
        wins.append((torch.randn(1, WIN, HKV, D, device=dev, generator=g).half(),
                     torch.randn(1, WIN, HKV, D, device=dev, generator=g).half()))
        del k, v
    qs = torch.randn(args.layers, 1, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    outs = torch.empty_like(qs)
    ws = torch.zeros(N.call("kvr_sd1_workspace_bytes", 1, HQ, HKV, NT, TILE, KSEL, WIN, 0) + 256, dtype=torch.uint8,
                     device=dev)

    def step():
        for li in range(args.layers):
            K.sd1_decode_step(stores[li], qs[li], KSEL, wins[li][0], wins[li][1], WIN, out=outs[li], ws=ws)

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        step()
        step()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(3):
            gr.replay()
        e0.record(stream)
        for _ in range(20):
            gr.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    layer_us = e0.elapsed_time(e1) / 20 / args.layers * 1e3

    n_units_win = WIN // 64
    att_blocks_win = [s + (n_units_win + KSEL) * h for h in range(HKV) for s in range(n_units_win)]
    att_blocks_tile = [s + (n_units_win + KSEL) * h for h in range(HKV) for s in range(n_units_win, n_units_win + KSEL)]
    rows = {}

    def add(name, v):
        rows.setdefault(name, []).append(v)

    if not args.split:
        cluster_phases(lib, gr, stream, args.reps, layer_us, args.layers)
        return
    for _ in range(args.reps):
        with torch.cuda.stream(stream):
            gr.replay()
        torch.cuda.synchronize()
        bs, ba = read(rd_sel), read(rd_att)
        sel_blocks = [b for b in range(SLOTS) if bs[(0 * SLOTS + b) * 8 + 0]]
        t0 = min(stamps(bs, 0, sel_blocks, 0))
        us = lambda x: (x - t0) / 1e3  # noqa: E731
        add("select: first CTA starts", us(min(stamps(bs, 0, sel_blocks, 0))))
        add("select: last CTA starts", us(max(stamps(bs, 0, sel_blocks, 0))))
        add("select: q' formed (last CTA)", us(max(stamps(bs, 0, sel_blocks, 1))))
        sc_end = stamps(bs, 0, sel_blocks, 2)
        if sc_end:
            add("select: tile scan done (last CTA)", us(max(sc_end)))
        att_start = stamps(ba, 1, att_blocks_win + att_blocks_tile, 0)
        add("attend: first CTA starts", us(min(att_start)))
        add("attend: last CTA starts", us(max(att_start)))
        add("attend: window units staged (last)", us(max(stamps(ba, 1, att_blocks_win, 1))))
        add("attend: window units done (last)", us(max(stamps(ba, 1, att_blocks_win, 3))))
        add("attend: tile units pass the grid wait (first)", us(min(stamps(ba, 3, att_blocks_tile, 6))))
        add("attend: tile units pass the grid wait (last)", us(max(stamps(ba, 3, att_blocks_tile, 6))))
        add("attend: tile rank select starts (last)", us(max(stamps(ba, 3, att_blocks_tile, 4))))
        add("attend: tile rank select done (last)", us(max(stamps(ba, 3, att_blocks_tile, 5))))
        add("attend: tile units staged (last)", us(max(stamps(ba, 1, att_blocks_tile, 1))))
        add("attend: tile units done (last)", us(max(stamps(ba, 1, att_blocks_tile, 3))))
        # merge stamps: only the CTA that arrives last for its head writes them;
        # other slots hold older layers' stamps, so take the latest per head
        allb = att_blocks_win + att_blocks_tile
        per = n_units_win + KSEL
        for pt, name in ((4, "merge starts"), (0, "merge: partial (m, l) loaded / weights formed"),
                         (1, "merge: partial halves staged"), (6, "merge: slots combined"),
                         (5, "merge done")):
            kern = 3 if pt in (0, 1) else 1
            heads = []
            for h in range(HKV):
                v = stamps(ba, kern, [b for b in allb if b // per == h], pt)
                if v:
                    heads.append(max(v))
            if heads:
                add(f"attend: {name} (first head)", us(min(heads)))
                add(f"attend: {name} (last head)", us(max(heads)))
    print(f"graph-replayed step: {layer_us:.2f} us per layer ({args.layers} layers)\n")
    print("| phase (last layer of the step) | us from the layer's first selection stamp (median) |")
    print("|---|---|")
    for name, vals in rows.items():
        print(f"| {name} | {statistics.median(vals):.2f} |")


if __name__ == "__main__":
    main()
