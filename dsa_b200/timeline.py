"""Device timeline of the config-4 decode step, and the key stream's read ceiling.

    python -m dsa_b200.build --timeline && python -m dsa_b200.timeline

Runs on the measurement build ``libtdsa_timeline.so`` (TDSA_TIMELINE defined: one thread
per CTA of the query projection, the dense score and the top-k records %globaltimer at
fixed points; the product library has none of it).  The workload is config 4's layer chain
-- per layer the fused query projection, the dense score with its key histogram and the
unsorted top-2048, 64 sequences of 32768 bf16 keys, 8 layers, random weights and keys --
issued as the bench issues it (eager launches, each a dependent launch on the previous
kernel).  For every layer it reports, as medians over layers and steps:

- the hand-offs between kernels (the last CTA of one kernel leaving -> the first CTA of the
  next passing its dependency wait);
- inside the projection: first ring stage landed, first refilled stage landed, last MMA
  issued, GEMM complete, the peer's partial sums received, exit (median CTA; exit the last);
- inside the score: last key tile issued (median CTA), exit (last CTA);
- inside the top-k: row copy landed, classification pass done (thread 0; median, 75th
  percentile and slowest row), candidate list written, k-th key found, output written
  (median row; and the last row).

``--no-projection`` issues the chain without the query projection (run once before, so
that every layer has its queries): score and top-k only, to see each one without the
projection's launches beside it.

Then the read ceiling of the same key bytes: the score kernel's key-tile stream with no
arithmetic (a 4-stage ring per SM of two 64-column swizzled boxes per tile, as the score
kernel loads them, or one plain bulk copy per tile), against the score kernel itself
launched back to back in a CUDA graph, over 8 rotating caches (no L2 reuse).
"""

from __future__ import annotations

import argparse
import ctypes as C
import statistics as S

import torch

from . import _capi as capi
from .build import LIB_TIMELINE

SLOTS = {"proj": (128, 8), "score": (148, 4), "topk": (64, 7)}


def _reader(lib, name):
    ncta, nslot = SLOTS[name]
    fn = getattr(lib, f"tdsa_timeline_{name}")
    arr = (C.c_ulonglong * (8 * ncta * nslot))()
    tickets = C.c_uint(0)

    def read():
        if fn(arr, C.byref(tickets)) != 0:
            raise RuntimeError(f"tdsa_timeline_{name} failed")
        return list(arr), tickets.value
    return read


def _launch_rows(arr, tickets, name, launch):
    """The records of launch `launch` (0 = the first launch after `tickets` was read)."""
    ncta, nslot = SLOTS[name]
    e = (tickets // ncta + launch) & 7
    return [arr[(e * ncta + c) * nslot:(e * ncta + c + 1) * nslot] for c in range(ncta)]


def chain(layers: int, batch: int, length: int, steps: int, device: torch.device,
          projection: bool = True) -> dict:
    from .indexer import ScoreTopkPlan
    from .sidecar import QueryProjector

    if batch != 64 or length != 32768:
        raise ValueError("the timeline records 64 top-k rows and 148 score CTAs: batch 64, "
                         "length 32768")
    hidden, k = 2048, 2048
    g = torch.Generator(device=device).manual_seed(5)
    std = hidden ** -0.5
    wq = [(torch.randn(8192, hidden, device=device, generator=g) * std).to(torch.bfloat16)
          for _ in range(layers)]
    ww = [torch.randn(64, hidden, device=device, generator=g) * std for _ in range(layers)]
    keys = [torch.randn(batch, length, 128, device=device, generator=g).to(torch.bfloat16)
            for _ in range(layers)]
    x = torch.randn(layers, batch, hidden, device=device, generator=g).to(torch.bfloat16)
    pos = torch.full((batch,), length - 1, device=device, dtype=torch.long)
    proj = [QueryProjector(wq[i], ww[i], batch) for i in range(layers)]
    plans = [ScoreTopkPlan(proj[i].q, proj[i].w, keys[i], k) for i in range(layers)]

    for i in range(layers):
        proj[i].project(x[i], pos)

    def step():
        for i in range(layers):
            if projection:
                proj[i].project(x[i], pos)
            plans[i].score()
            plans[i].select()

    for _ in range(5):
        step()
    torch.cuda.synchronize(device)
    lib = capi.lib()
    rd = {name: _reader(lib, name) for name in SLOTS}
    seg: dict[str, list[float]] = {}

    def add(name, v_ns):
        seg.setdefault(name, []).append(v_ns / 1e3)

    for _ in range(steps):
        tick = {name: rd[name]()[1] for name in SLOTS}
        step()
        torch.cuda.synchronize(device)
        arr = {name: rd[name]()[0] for name in SLOTS}
        prev_end = None
        for i in range(layers):
            s = _launch_rows(arr["score"], tick["score"], "score", i)
            t = _launch_rows(arr["topk"], tick["topk"], "topk", i)
            s_wait = min(r[1] for r in s)
            s_exit = max(r[3] for r in s)
            t_wait = min(r[1] for r in t)
            t_end = max(r[5] for r in t)
            if prev_end is not None:
                add("layer (top-k end to top-k end)", t_end - prev_end)
            if projection:
                p = _launch_rows(arr["proj"], tick["proj"], "proj", i)
                p_wait = min(r[1] for r in p)
                p_exit = max(r[7] for r in p)
                if prev_end is not None:
                    add("hand-off top-k -> projection", p_wait - prev_end)
                for j, name in ((2, "first stage landed"), (3, "first refilled stage landed"),
                                (4, "last MMA issued"), (5, "GEMM complete"),
                                (6, "peer partial sums received")):
                    add(f"projection: wait -> {name}", S.median(r[j] - r[1] for r in p))
                add("projection: wait -> exit (last CTA)", p_exit - p_wait)
                add("hand-off projection -> score", s_wait - p_exit)
            add("score: wait -> last key tile issued", S.median(r[2] - r[1] for r in s))
            add("score: wait -> exit (last CTA)", s_exit - s_wait)
            add("score: exit spread (last - first CTA)",
                s_exit - min(r[3] for r in s))
            add("hand-off score -> top-k", t_wait - s_exit)
            classify = sorted(r[6] - r[2] for r in t)
            add("top-k: row copy landed -> classification done", S.median(classify))
            add("top-k: ... (75th percentile row)", classify[(3 * len(classify)) // 4])
            add("top-k: ... (slowest row)", classify[-1])
            for j, name in ((2, "row copy landed"), (3, "candidate list written"),
                            (4, "k-th key found"), (5, "output written")):
                add(f"top-k: wait -> {name}", S.median(r[j] - r[1] for r in t))
            add("top-k: wait -> output written (last row)", t_end - t_wait)
            prev_end = t_end
    return {name: S.median(v) for name, v in seg.items()}


def read_ceiling(batch: int, length: int, device: torch.device, ncache: int = 8) -> dict:
    from .indexer import ScoreTopkPlan

    lib = capi.lib()
    g = torch.Generator(device=device).manual_seed(6)
    caches = [torch.randn(batch, length, 128, device=device, generator=g).to(torch.bfloat16)
              for _ in range(ncache)]
    nbytes = batch * length * 256
    stream = torch.cuda.current_stream(device)

    def timed(fn, reps=24, skip=8):
        ts = []
        for r in range(reps):
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(stream)
            fn(r % ncache)
            b.record(stream)
            torch.cuda.synchronize(device)
            if r >= skip:
                ts.append(a.elapsed_time(b) * 1e3)
        return S.median(ts)

    out = {}
    for mode, name in ((0, "ring, two 64-column swizzled boxes per tile (score's loads)"),
                       (1, "ring, one plain bulk copy per tile")):
        def run(i, mode=mode):
            capi.check(lib.tdsa_timeline_read_stream(C.c_void_p(caches[i].data_ptr()), batch,
                                                     length, mode,
                                                     C.c_void_p(stream.cuda_stream)))
        us = timed(run)
        out[name] = (us, nbytes / us / 1e3)
    q = (torch.randn(batch, 64, 128, device=device, generator=g) / 128 ** 0.5).to(
        torch.bfloat16)
    w = torch.randn(batch, 64, device=device, generator=g) / 8
    plans = [ScoreTopkPlan(q, w, c, 2048) for c in caches]
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for p in plans:
            p.score()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for p in plans:
            p.score()
    ts = []
    for _ in range(15):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize(device)
        ts.append(a.elapsed_time(b) * 1e3 / ncache)
    del graph
    us = S.median(ts)
    out["score kernel, back to back in a CUDA graph"] = (us, nbytes / us / 1e3)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--length", type=int, default=32768)
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--no-projection", action="store_true",
                    help="score and top-k only (the projection runs once, before)")
    args = ap.parse_args()
    if not LIB_TIMELINE.exists():
        raise SystemExit(f"{LIB_TIMELINE} is missing: python -m dsa_b200.build --timeline")
    capi.LIB_PATH = LIB_TIMELINE  # before the first library call
    device = torch.device("cuda", torch.cuda.current_device())
    res = chain(args.layers, args.batch, args.length, args.steps, device,
                projection=not args.no_projection)
    what = "score + top-k only" if args.no_projection else "project, score, top-k"
    print(f"config-4 layer chain ({what}), batch {args.batch}, {args.length} keys, "
          f"{args.layers} layers, medians over {args.steps} steps (us)")
    for name, v in res.items():
        print(f"  {name:48s} {v:8.2f}")
    if not args.no_projection:
        print("key stream of one score launch "
              f"({args.batch * args.length * 256 / 1e6:.1f} MB), 8 rotating caches (us, GB/s)")
    if not args.no_projection:
        for name, (us, gbs) in read_ceiling(args.batch, args.length, device).items():
            print(f"  {name:64s} {us:8.2f} {gbs:8.0f}")
    status = capi.device_status(True)
    print(f"device status {status}")
    if status:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
