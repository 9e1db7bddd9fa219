"""The independent work of the hot path, sharded over the GPUs of one node
(test infrastructure: one process per GPU, launched by torchrun).

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P tests/multi_gpu.py [--what sweep,cases] [--out FILE]

* sweep (Tests/OpTests.lean:273-296): rank r maps
  its contiguous share of the 2^32 binary32 bit patterns (shard.sweep_range)
  through the GPU's erff_map in chunks of 2^24 and compares each chunk on the
  device (`binary ne`, then `count_nonzero`, as the reference does) with the
  oracle's correctly rounded erff computed on this rank's share of the host
  cores. The mismatch counts are summed over the ranks; the planted fault (the
  CPU side one input late) must differ on every rank.
* cases (Tests/OpTests.lean:361-381): the 38 ggml cases dealt round robin
  (shard.round_robin); each rank runs its cases through the executor,
  compiled and uncompiled, compares the output's SHA-256 with the reference's
  pin, runs the planted wrong lowering (which must differ or refuse) and the
  refusals; the results are gathered to rank 0.

Rank 0 prints one JSON line per part (and writes them to --out). The control
plane is gloo; no kernel reads another GPU's memory.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import datetime
import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "contract-stablehlo-mlx_b200"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        return 0, 0, 1, None
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    return dist.get_rank(), int(os.environ.get("LOCAL_RANK", "0")), ws, dist


def sweep(rank, ws, dist, M, Run, O, S, chunk_log=24):
    lo, hi = S.sweep_range(ws, rank)
    chunks = S.sweep_chunks(lo, hi, 1 << chunk_log)
    threads = max(1, (os.cpu_count() or 1) // ws)
    bad, first_bad, gpu_s = 0, None, 0.0
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        futs = {ex.submit(O.erff_range, b, n, 1): (b, n) for b, n in chunks}
        for fut in cf.as_completed(futs):
            b, n = futs[fut]
            g0 = time.perf_counter()
            gpu = Run.erff_map(b, n)
            M.eval_([gpu])
            gpu_s += time.perf_counter() - g0
            cpu = M.of_numpy(fut.result(), M.dtU32)
            k = M.count_nonzero(M.binary(M.opNe, gpu, cpu))
            if k:
                bad += k
                first_bad = b if first_bad is None else min(first_bad, b)
    dt = time.perf_counter() - t0
    # the planted fault: the CPU side one input late must differ, on a window
    # where erff varies (a rank's own share may lie where it is +-1 throughout)
    b0, n0 = 0x3F000000, 1 << 20
    planted = M.count_nonzero(M.binary(M.opNe, Run.erff_map(b0, n0), M.of_numpy(O.erff_range(b0 + 1, n0), M.dtU32)))
    total = S.sum_over_ranks(dist, bad)
    caught = S.sum_over_ranks(dist, 1 if planted else 0)
    firsts = [first_bad]
    if dist is not None:
        firsts = [None] * ws
        dist.all_gather_object(firsts, first_bad)
    e2e = S.max_over_ranks(dist, dt)
    gmax = S.max_over_ranks(dist, gpu_s)
    return {"what": "erf-sweep", "n_gpus": ws, "patterns": S.SWEEP_PATTERNS,
            "mismatches": total, "first_mismatch_chunk": min([f for f in firsts if f is not None], default=None),
            "planted_fault_caught_on_ranks": caught, "host_threads_per_rank": threads,
            "gpu_map_s": round(gmax, 3), "e2e_s": round(e2e, 3),
            "gpu_patterns_per_s": round(S.SWEEP_PATTERNS / gmax, 1),
            "e2e_patterns_per_s": round(S.SWEEP_PATTERNS / e2e, 1),
            "note": "gpu_map_s: the slowest rank's erff_map time (launch to eval), e2e_s: the slowest rank's whole "
                    "share including the host oracle, both max over ranks"}


def cases(rank, ws, dist, M, S):
    import optests as T
    from oracle import ggml_cases as G
    from shlo import exec as E
    from shlo import lower as L
    from conftest import load_pins

    pins = load_pins("pinned")

    def run_module(text, ins, faults, compile):
        try:
            outs = E.call(E.prepare(E.load(text), faults, compile), ins)
            return "ok", M.to_bytes(outs[0])
        except M.ShloError as e:
            return "err", str(e)

    mine = S.round_robin(T.cases(), ws, rank)
    results = []
    t0 = time.perf_counter()
    for oc in mine:
        c = G.BY_NAME[oc.name]
        ins = [M.of_numpy(a) for a in c.inputs()]
        ins_ne = [ne for ne, _ in c.ins]
        text = T.view_module(ins_ne[0], c.out_ne, oc.view_offset) if oc.op == "view" else \
            T.module_for(oc.op, ins_ne, c.out_ne)
        want = pins["%s/out.f32" % oc.name]
        ok, why = True, ""
        if oc.expect_refusal:
            st, msg = run_module(text, ins, L.Faults(), True)
            ok = st == "err" and "not carried" in msg
            why = "" if ok else "not refused: %s" % msg[:100]
        else:
            for compile in (True, False):
                st, got = run_module(text, ins, L.Faults(), compile)
                if st != "ok" or hashlib.sha256(got).hexdigest() != want:
                    ok, why = False, "%s: %s" % ("compiled" if compile else "uncompiled",
                                                 got[:100] if st != "ok" else "hash differs")
                    break
            fault = oc.fault
            if fault.dotPlain and c.extra["K"] < 16:
                fault = L.Faults(dotBuiltin=True)  # the pinned tail equals the planted sum below K = 16
            st, got = run_module(text, ins, fault, True)
            if ok and st == "ok" and hashlib.sha256(got).hexdigest() == want:
                ok, why = False, "planted fault (%s) not caught" % oc.fault_name
        results.append((oc.name, rank, ok, why))
    dt = time.perf_counter() - t0
    allres = [results]
    if dist is not None:
        allres = [None] * ws
        dist.all_gather_object(allres, results)
    flat = [r for part in allres for r in part]
    e2e = S.max_over_ranks(dist, dt)
    failed = [(n, r, why) for n, r, ok, why in flat if not ok]
    return {"what": "op-cases", "n_gpus": ws, "cases": len(flat), "passed": len(flat) - len(failed),
            "failed": failed, "per_rank": [sum(1 for _, r, _, _ in flat if r == k) for k in range(ws)],
            "wall_s_max_over_ranks": round(e2e, 2)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", default="sweep,cases")
    ap.add_argument("--out", default="")
    ap.add_argument("--chunk-log", type=int, default=24)
    args = ap.parse_args()
    rank, local_rank, ws, dist = init()
    from oracle import oracle as O
    from shlo import mlx as M
    from shlo import run as Run
    from shlo import shard as S

    M.set_device(local_rank)
    M.set_flavor("pinned")
    lines = []
    for part in args.what.split(","):
        if part == "sweep":
            lines.append(sweep(rank, ws, dist, M, Run, O, S, args.chunk_log))
        elif part == "cases":
            lines.append(cases(rank, ws, dist, M, S))
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)
        if args.out:
            with open(args.out, "a") as f:
                for ln in lines:
                    f.write(json.dumps(ln) + "\n")
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    bad = any(ln.get("mismatches", 0) or ln.get("failed") for ln in lines) or \
        any(ln.get("planted_fault_caught_on_ranks", ws) != ws for ln in lines if ln["what"] == "erf-sweep")
    sys.exit(1 if bad else 0)


if __name__ == "__main__":
    main()
