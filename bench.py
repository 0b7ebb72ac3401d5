"""Decode throughput of the B200 engine on LAICompute's Llama decode loop.

Default workload: the SmolLM-135M-shaped Llama with Q8_0 projections (hidden
576, 30 layers, 9/3 heads, ffn 1536, vocab 49152, tied Q8_0 embeddings),
random-init from a fixed seed, 64 independent sequences, 128 random prompt
ids each, then decode steps. One "step" = one token for every sequence.

  value  tokens/s of K device-chained decode steps (laic_dev_decode: each step
         feeds every sequence its own sampled id without leaving the device),
         CUDA events on the engine stream, max over ranks
  e2e    tokens/s of K laic_dev_step calls (the C ABI a caller uses): host ids
         in through pinned memory, sampled ids back to the host, every step;
         the sequences start again from their prompts first, so both numbers
         cover the same positions

Multi-GPU (torchrun, one rank per GPU): the 135M model does not shard per
layer, so every rank decodes its own 64 sequences (replicas, weak scaling).

Two more measurements ride on the same line:
  llama8b_b1  the 8B-shaped Q4_0 model (tied Q4_0 lm_head), batch 1, prompt
              1024, KV cache of 8192 positions, split tensor-parallel over all
              the run's GPUs (peer-memory allreduce after o and down; strong
              scaling): tokens/s, ms per step, HBM GB/s of the weight + KV
              stream and its fraction of the measured copy peak, e2e
  c3_sweep    (rank 0) the Q4_0 matvec sweep: out x in = 1536x576, 576x1536,
              4096x4096, 14336x4096, 4096x14336, 128256x4096 at batch 1, 4, 16
              through laic_tensor_matvec, each launch timed with CUDA events
              after a write of 256 MB (twice the L2) that evicts the weights
--workload picks another headline workload (llama8b-q4_0 is then the headline).

--impl reference times the reference's own CPU decode loop (oracle/_ref, the
reference sources compiled with its native flags) on the same model and
prompt, one sequence at a time as the reference runs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from dataclasses import replace  # noqa: E402

from laicompute_b200 import synth  # noqa: E402

WORKLOADS = {
    # name: (arch, seed, prompt_len, batch, description)
    "smollm135m-q8_0": (synth.SMOL_135M_Q8, 2, 128, 64, "SmolLM-135M-shaped Llama, Q8_0 projections"),
    "smollm135m-f16": (synth.SMOL_135M_F16, 1, 8, 1, "SmolLM-135M-shaped Llama, F16"),
    "llama1b-q4_0": (synth.LLAMA_1B_Q4, 4, 512, 32, "1B-shaped Llama, Q4_0 projections, F16 embeddings"),
    "llama8b-q4_0": (synth.LLAMA_8B_Q4, 5, 1024, 1, "8B-shaped Llama, Q4_0 projections, tied Q4_0 embeddings"),
    # two layers of the 8B shape: the same kernels and launch shapes on ~0.5 GB of weights, the
    # small case for multi-pass profiler captures of the 8B kernels
    "llama8b-2l-q4_0": (replace(synth.LLAMA_8B_Q4, name="llama-8b-2l-q4_0", layers=2), 5, 1024, 1,
                        "two layers of the 8B-shaped Llama (profiling case)"),
}
# workloads split tensor-parallel over the GPUs of the run (the others run one replica per GPU)
TP_WORKLOADS = {"llama8b-q4_0"}
# KV positions allocated per slot, where the workload asks for more than it decodes
KV_CAPACITY = {"llama8b-q4_0": 8192, "llama8b-2l-q4_0": 8192}
# CPU sample of the large models: (prompt tokens, timed decode steps) — a reference step takes seconds
CPU_SAMPLE = {"llama1b-q4_0": (64, 16), "llama8b-q4_0": (32, 8)}
DEFAULT_WORKLOAD = "smollm135m-q8_0"


def measured_peak_gbs():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def model_path(name: str, rank: int) -> str:
    """The workload's GGUF (rank = None: one file shared by the ranks of a tensor-parallel run)."""
    arch, seed, _, _, _ = WORKLOADS[name]
    d = os.path.join(tempfile.gettempdir(), "laic_bench_models")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{name}.seed{seed}" + ("" if rank is None else f".r{rank}") + ".gguf")
    if not os.path.exists(path):
        tmp = path + ".part"
        # quantised tensors of the large models are drawn as random blocks (quantising 8B values takes minutes)
        synth.write_model(tmp, arch, seed=seed, direct_blocks=arch.hidden >= 2048)
        os.replace(tmp, path)
    return path


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples of one GPU during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str) -> None:
        self.uuid = uuid
        self.rows = []
        self.proc = None
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 3.0:  # nvidia-smi takes a moment to start
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_reference(name: str, path: str, warmup: int, steps: int) -> dict:
    """The reference's CPU decode loop on one sequence (oracle/_ref, native flags)."""
    from oracle import oracle as O
    arch, seed, plen, _, _ = WORKLOADS[name]
    if name in CPU_SAMPLE:
        plen, steps = CPU_SAMPLE[name][0], min(steps, CPU_SAMPLE[name][1])
    prompt = synth.prompt_ids(arch.vocab, plen, seed=seed + 100)
    exe, kind = None, "reference"
    for variant in ("native", "v3"):
        cand = O.ref_driver(variant)
        if cand and subprocess.run([cand], capture_output=True).returncode == 2:  # usage exit: runs on this CPU
            exe = cand
            break
    if exe is None:
        return {"unavailable": "reference driver not built or not runnable on this CPU"}
    with tempfile.NamedTemporaryFile(suffix=".u32", delete=False) as f:
        prompt.tofile(f.name)
        pf = f.name
    try:
        r = subprocess.run([exe, "time", path, "--prompt", pf, "--warmup", str(warmup), "--steps", str(steps)],
                           capture_output=True, text=True, check=True)
    finally:
        os.unlink(pf)
    info = json.loads(r.stdout.strip().splitlines()[-1])
    return {"value": info["tok_s"], "unit": "tokens/s", "cores": info["threads"], "kind": kind,
            "sample": f"{os.path.basename(exe)}: {plen}-token prompt (untimed), {warmup} warm-up + {steps} timed "
                      f"decode steps of one sequence on {info['threads']} threads (the reference decodes one "
                      f"sequence at a time, so its tokens/s does not depend on the batch)",
            "prefill_s": info["prefill_s"], "steps": steps}


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    name = args.workload
    arch, seed, plen, batch, desc = WORKLOADS[name]
    path = model_path(name, 0)
    steps = min(args.steps, args.ref_steps)
    res = cpu_reference(name, path, max(1, min(args.warmup, 3)), steps)
    if "unavailable" in res:
        print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}))
        return
    out = {
        "impl": "reference", "metric": "decode tokens/s", "value": round(res["value"], 3), "unit": "tokens/s",
        "n_gpus": world, "steps": res["steps"], "warmup": args.warmup, "ms_per_step": round(1000.0 / res["value"], 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{name} decode", "model": desc, "batch": batch, "prompt": plen,
                   "note": "reference CPU loop, one sequence at a time"},
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(res["value"], 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def allgather_floats(x: float, world: int) -> list:
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(v.item()) for v in out]


def gpu_uuid(local: int) -> str:
    import torch
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    return uuid if uuid.startswith("GPU-") else "GPU-" + uuid


def run_decode(name: str, args, world: int, rank: int, local: int, batch: int, sample: bool,
               clocks: bool) -> dict:
    """Build the workload's engine, prefill every sequence, then time K chained decode
    steps (value) and K host-in/host-out steps (e2e); returns the measurements (every rank)."""
    import torch
    from laicompute_b200.engine import Engine, nccl_unique_id, sample_params

    arch, seed, plen, _, desc = WORKLOADS[name]
    tp = world if (name in TP_WORKLOADS and world > 1) else 1
    if tp > 1:  # one model file, written by rank 0; the ranks hold shards of one engine
        if rank == 0:
            path = model_path(name, None)
        barrier(world)
        path = model_path(name, None)
        nid = [nccl_unique_id() if rank == 0 else None]
        import torch.distributed as dist
        dist.broadcast_object_list(nid, src=0, device=torch.device("cuda", local))
        tp_kw = dict(tp_size=tp, tp_rank=rank, nccl_id=nid[0])
    else:
        path = model_path(name, rank)
        tp_kw = {}
    seq_rank = 0 if tp > 1 else rank  # tensor-parallel ranks decode the same sequences
    ctx_need = plen + 2 * args.warmup + 2 * args.steps + 64  # decode, e2e and profiling steps
    ctx_need = max(ctx_need, KV_CAPACITY.get(name, 0))
    eng = Engine(path, max_seqs=batch, device=local, kv_capacity=ctx_need, layer_launches=args.layer_launches,
                 step_kernel=True if args.step_kernel else None, **tp_kw)
    slots = np.arange(batch, dtype=np.int32)
    prompts = np.stack([synth.prompt_ids(arch.vocab, plen, seed=seed + 100 + 1000 * seq_rank + i)
                        for i in range(batch)])
    if sample:
        params = [sample_params(0.8, 40, 1.0, 1.0, 4242 + 1000 * seq_rank + i) for i in range(batch)]
    else:
        params = [sample_params()] * batch

    def start_sequences():
        """Every slot from empty: the prompts (all but their last token) in batched passes,
        then the first decode step; returns that step's ids and the prefill seconds."""
        for i in range(batch):
            eng.reset_slot(int(slots[i]))
        torch.cuda.synchronize()
        t_pf = time.perf_counter()
        for i in range(batch):
            eng.prefill_batch(prompts[i, :-1], int(slots[i]))
        eng.sync()
        pf_s = time.perf_counter() - t_pf
        ids0, _ = eng.step(prompts[:, -1], slots, params)
        return ids0, pf_s

    first, prefill_s = start_sequences()  # the prefill is timed as a side figure

    # ---- device-resident decode loop (value), clocks sampled from before it to after the e2e loop
    ids_w, _ = eng.decode(first, slots, params, steps=args.warmup)
    tok = ids_w[-1]
    clk = ClockSampler(gpu_uuid(local)) if clocks else None
    if clk:
        clk.__enter__()
    barrier(world)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()  # marks the timed region for `ncu --profile-from-start off`
    ids, dev_ms = eng.decode(tok, slots, params, steps=args.steps)
    torch.cuda.profiler.stop()
    barrier(world)
    torch.cuda.synchronize()
    rank_ms = allgather_floats(dev_ms, world)
    max_ms = max(rank_ms)
    replicas = world // tp  # independent sequence batches in the job
    value = batch * args.steps * replicas / (max_ms / 1000.0)
    launches_chained = eng.stats().launches_per_step  # kernels per chained step, as timed

    # ---- end to end through laic_dev_step: host ids in, sampled ids out, every step, over the
    #      same positions as the device-resident loop (the sequences start again from the prompt)
    local_dev = torch.device("cuda", local)
    ext = torch.cuda.ExternalStream(eng.stream, device=local_dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tok, _ = start_sequences()
    for _ in range(args.warmup):
        tok, _ = eng.step(tok, slots, params)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(ext)
    for _ in range(args.steps):
        tok, _ = eng.step(tok, slots, params)
    e1.record(ext)
    e1.synchronize()
    if clk:
        clk.__exit__(None, None, None)
    e2e_ms = allreduce_max(e0.elapsed_time(e1), world)
    e2e_value = batch * args.steps * replicas / (e2e_ms / 1000.0)

    # ---- per-kernel roofline (eager launches with CUDA events around each)
    st = eng.stats()
    prof = eng.profile(np.tile(tok, 4), 4)
    eng.close()
    peak, peak_kind = measured_peak_gbs()
    dname, (dl, dus, dbytes) = max(prof.items(), key=lambda kv: kv[1][1])
    achieved = (dbytes / dl) / (dus / dl * 1e-6) / 1e9
    traffic = None  # DRAM bytes per launch: ncu's bytes per algorithmic byte (profiles/traffic.json) x ours
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            ratio = json.load(f).get(name, {}).get(dname)
        if ratio:
            traffic = int(round(ratio * dbytes / dl))
    except (OSError, ValueError):
        pass
    # KV bytes read per step in the timed decode: every sequence reads its whole context (all layers, K+V)
    mid_pos = plen + args.warmup + args.steps / 2.0
    kv_read = st.kv_bytes_per_pos * batch * mid_pos
    step_s = max_ms / args.steps * 1e-3
    step_gbs = (st.weight_bytes + kv_read) / step_s / 1e9
    return {
        "name": name, "desc": desc, "tp": tp, "batch": batch, "plen": plen, "value": value, "max_ms": max_ms,
        "rank_ms": rank_ms, "e2e_value": e2e_value, "launches": launches_chained, "prefill_s": prefill_s,
        "weight_bytes": st.weight_bytes, "kv_read": kv_read, "step_gbs": step_gbs, "peak": peak,
        "peak_kind": peak_kind, "clocks": clk.summary() if clk else None,
        "roofline": {"bound": "hbm", "kernel": dname, "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                     "bytes_per_launch": round(dbytes / dl), "us_per_launch": round(dus / dl, 3),
                     "timing": "eager launches of 4 full steps, CUDA events around each launch",
                     "kernels": {k: {"launches": v[0], "us_per_launch": round(v[1] / v[0], 3),
                                     "gbs": round(v[2] / v[1] * 1e-3, 1)} for k, v in prof.items()}},
        "step_roofline": {"bound": "hbm", "kernel": "decode step (graph replay)", "achieved": round(step_gbs, 1),
                          "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(step_gbs / peak, 4),
                          "bytes_per_step": int(st.weight_bytes + kv_read), "us_per_step": round(step_s * 1e6, 3)},
    }


SWEEP_SHAPES = [(1536, 576), (576, 1536), (4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


def run_sweep(local: int, launches: int = 20) -> dict:
    """The Q4_0 matvec sweep through laic_tensor_matvec with a cold L2 before every launch."""
    import torch
    from laicompute_b200 import gguf
    from laicompute_b200.engine import Matrix
    peak, peak_kind = measured_peak_gbs()
    dev = torch.device("cuda", local)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    rows = []
    for out_dim, in_dim in SWEEP_SHAPES:
        rng = np.random.default_rng(out_dim * 7 + in_dim)
        raw = np.frombuffer(synth.random_blocks(out_dim * in_dim, gguf.Q4_0, rng), dtype=np.uint8)
        m = Matrix(gguf.Q4_0, in_dim, out_dim, raw, device=local)
        x = torch.from_numpy(rng.standard_normal((16, in_dim), dtype=np.float32)).to(dev)
        y = torch.empty((16, out_dim), dtype=torch.float32, device=dev)
        for batch in (1, 4, 16):
            for _ in range(3):
                m.matvec(x.data_ptr(), y.data_ptr(), batch, stream.cuda_stream)
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(launches)]
            for a, b in ev:
                flush.fill_(1)  # 256 MB written: the matrix is no longer in L2
                a.record(stream)
                m.matvec(x.data_ptr(), y.data_ptr(), batch, stream.cuda_stream)
                b.record(stream)
            torch.cuda.synchronize(dev)
            us = statistics.median(a.elapsed_time(b) * 1000.0 for a, b in ev)
            nbytes = m.nbytes + 4 * batch * (in_dim + out_dim)
            gbs = nbytes / (us * 1e-6) / 1e9
            rows.append({"out": out_dim, "in": in_dim, "batch": batch, "us": round(us, 3), "bytes": nbytes,
                         "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})
        m.check(stream.cuda_stream)
        m.close()
    return {"kernel": "laic_tensor_matvec (Q4_0)", "timing": f"median of {launches} launches, CUDA events, "
                                                              "L2 flushed by a 256 MB write before each",
            "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "rows": rows}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="sequences per GPU (0 = the workload's)")
    ap.add_argument("--sample", action="store_true", help="temperature 0.8 / top-k 40 instead of greedy")
    ap.add_argument("--ref-steps", type=int, default=64, help="cap of timed CPU decode steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true")
    ap.add_argument("--no-llama8b", action="store_true", help="skip the 8B batch-1 tensor-parallel measurement")
    ap.add_argument("--no-sweep", action="store_true", help="skip the Q4_0 matvec sweep")
    ap.add_argument("--layer-launches", action="store_true",
                    help="one sequence: always per-layer launches, never the persistent decode-step kernel")
    ap.add_argument("--step-kernel", action="store_true",
                    help="one sequence: always the persistent decode-step kernel (default: the engine's choice "
                         "by layer size)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    world, rank, local = dist_setup()
    import torch
    from laicompute_b200.engine import Engine

    name = args.workload
    arch, seed, plen, batch, desc = WORKLOADS[name]
    if args.batch:
        batch = args.batch
    r = run_decode(name, args, world, rank, local, batch, args.sample, clocks=rank == 0)
    out = None
    if rank == 0:
        spread = (max(r["rank_ms"]) - min(r["rank_ms"])) / max(r["rank_ms"])
        out = {
            "metric": "decode tokens/s", "value": round(r["value"], 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["max_ms"] / args.steps, 5),
            "higher_is_better": True, "scaling": "strong" if r["tp"] > 1 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{name} decode, batch {batch} per GPU, prompt {plen}, "
                                   f"{'T=0.8/top-k 40' if args.sample else 'greedy'}",
                       "model": desc, "batch_per_gpu": batch, "prompt": plen,
                       "parallelism": f"tp{r['tp']}" if r["tp"] > 1 else f"replicas x{world}", "kv": "fp16",
                       "l2": "inputs larger than L2: weights %.0f MB + KV read %.0f MB per step"
                             % (r["weight_bytes"] / 1e6, r["kv_read"] / 1e6)},
            "hbm_gbs_step": round(r["step_gbs"], 1),
            "rank_ms_per_step": [round(v / args.steps, 5) for v in r["rank_ms"]],
            "rank_spread": round(spread, 4),
            "e2e": {"value": round(r["e2e_value"], 2), "unit": "tokens/s", "h2d_bytes_per_step": batch * (4 + 4 + 24),
                    "d2h_bytes_per_step": batch * 4 + 8},
            "gpu_launches": int(args.steps * r["launches"]),
            "prefill": {"tokens_per_s": round(batch * (plen - 1) / r["prefill_s"], 1), "prompt_tokens": plen - 1,
                        "sequences": batch, "batched": r["tp"] == 1,
                        "timing": "host wall clock, engine synchronised"},
            "roofline": r["roofline"],
            "step_roofline": r["step_roofline"],
            "clocks": r["clocks"],
        }

    # ---- batch-1 decode (the latency case) on the same model
    if not args.no_batch1 and batch > 1:
        path = model_path(name, rank)
        ctx_need = plen + 2 * args.warmup + 2 * args.steps + 64
        e1b = Engine(path, max_seqs=1, device=local, kv_capacity=ctx_need)
        prompt = synth.prompt_ids(arch.vocab, plen, seed=seed + 100 + 1000 * rank)
        e1b.prefill_batch(prompt[:-1], 0)
        f1, _ = e1b.step([prompt[-1]], [0])
        w, _ = e1b.decode(f1, [0], None, steps=args.warmup)
        barrier(world)
        _, ms1 = e1b.decode(w[-1], [0], None, steps=args.steps)
        ms1 = allreduce_max(ms1, world)
        if out is not None:
            s1 = e1b.stats()
            out["batch1"] = {"value": round(args.steps * world / (ms1 / 1000.0), 2), "unit": "tokens/s",
                             "ms_per_step": round(ms1 / args.steps, 5),
                             "hbm_gbs": round(s1.weight_bytes / (ms1 / args.steps * 1e-3) / 1e9, 1)}
        e1b.close()

    # ---- the 8B-shaped model at batch 1, tensor-parallel over every GPU of the run
    if not args.no_llama8b and name != "llama8b-q4_0":
        r8 = run_decode("llama8b-q4_0", args, world, rank, local, 1, False, clocks=rank == 0)
        if out is not None:
            out["llama8b_b1"] = {
                "workload": "llama8b-q4_0 decode, batch 1, prompt 1024, KV capacity 8192, greedy",
                "parallelism": f"tp{r8['tp']}" if r8["tp"] > 1 else "single GPU", "tokens_per_s": round(r8["value"], 2),
                "ms_per_step": round(r8["max_ms"] / args.steps, 5),
                "rank_ms_per_step": [round(v / args.steps, 5) for v in r8["rank_ms"]],
                "hbm_gbs": round(r8["step_gbs"], 1),
                "frac": round(r8["step_gbs"] / r8["peak"], 4), "peak": r8["peak"], "peak_kind": r8["peak_kind"],
                "bytes_per_step": int(r8["weight_bytes"] + r8["kv_read"]),
                "bytes_note": "weights of every rank's shard (this rank's bytes x ranks for the GB/s of the job) "
                              "+ KV read" if r8["tp"] > 1 else "weights + KV read",
                "e2e": {"value": round(r8["e2e_value"], 2), "unit": "tokens/s"},
                "gpu_launches_per_step": r8["launches"],
                "roofline": r8["roofline"], "clocks": r8["clocks"],
            }
            if r8["tp"] > 1:  # the job streams every rank's shard in one step
                job_gbs = r8["step_gbs"] * r8["tp"]
                out["llama8b_b1"]["hbm_gbs_job"] = round(job_gbs, 1)
                out["llama8b_b1"]["frac_job"] = round(job_gbs / (r8["peak"] * r8["tp"]), 4)

    # ---- the Q4_0 matvec sweep (rank 0)
    if not args.no_sweep and rank == 0:
        out["c3_sweep"] = run_sweep(local)
    barrier(world)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res = cpu_reference(name, model_path(name, rank), 1, min(args.steps, 16))
        if "unavailable" not in res:
            out["cpu_baseline"] = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")}
        else:
            out["cpu_baseline"] = None
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
