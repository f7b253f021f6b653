"""Benchmark: int4-g32-a16 GPT-2 124M batch-1 greedy decode (config 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one whole config-0 generation: prompt [50256], then 100 greedy
tokens (100 model forwards, each one decode step of the int4-g32-a16
layers, the int8 per-channel head with its argmax, and the int8 KV cache).
Weights are random-init (N(0, 0.02), seed 0); no checkpoint is read.

value: generated tokens / device time of the K timed steps (CUDA events on
the library's stream, L2 flushed by a 256 MiB write between steps, prompt
and ids resident in HBM). e2e: the same through llmq_generate with host
prompt and host ids (the copies inside the timed region). roofline: the
dominant kernel (the persistent decode kernel, one launch per generation),
timed live with CUDA events on its stream, against the measured HBM copy
bandwidth. cpu_baseline: the CPU oracle (a C restatement of the reference's
path: a thread team of one thread per physical core, VNNI integer dots) on
a bounded sample. With N GPUs (torchrun), each rank decodes its own sequence
(replicas of the batch-1 decode, which does not shard), and value is the
sum over ranks with the max device time over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

STEPS_PER_GEN = 100
PROMPT = [50256]
HEAD_BYTES = 50257 * 768 + 50257 * 3          # int8-ch head: codes + f16 scale + u8 zp per row
LAYER_WEIGHTS = 12 * (768 * (2304 + 768 + 3072) + 3072 * 768)  # 84,934,656
LAYER_BYTES = LAYER_WEIGHTS * 19 // 32         # int4-g32: 0.59375 B/weight = 50,429,952
TOKEN_BYTES = LAYER_BYTES + HEAD_BYTES         # 89,178,099 per token
METRIC = "int4-g32-a16 decode tok/s (b=1)"
# DRAM bytes (read + write) of one persistent-kernel launch of this workload,
# from one ncu capture (profiles/mega_decode_kernel.txt): below the
# algorithmic bytes because the weight stream stays in L2 across tokens.
MEGA_TRAFFIC_BYTES = 4_058_159_360


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)  # the sampler is running before the timed region starts
            self.lines.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(seconds: float = 20.0, samples: int = 5):
    """The CPU oracle's greedy decode of config 0: `samples` runs (the prompt
    forward, then decode steps up to the 100-token generation or
    seconds / samples), tokens per second over the decode steps each
    finished; the median of the runs (five by default, as the reference's
    published CPU figure is a median of five)."""
    from llm_mojo_b200 import synth
    from oracle import oracle as O

    t = synth.gpt2_random_init(0)
    m = O.Model(t)
    rates, steps = [], []
    for _ in range(samples):
        logits = m.forward(PROMPT, 0)
        n, pos, t0 = 1, 1, time.perf_counter()
        while time.perf_counter() - t0 < seconds / samples and n < STEPS_PER_GEN:
            nxt = int(O.lib().oq_argmax(O.ptr(logits), m.V))
            logits = m.forward([nxt], pos)
            pos += 1
            n += 1
        rates.append((n - 1) / (time.perf_counter() - t0))
        steps.append(n - 1)
    m.close()
    threads = int(O.lib().oq_threads())
    vnni = bool(O.lib().oq_set_vnni(1))
    return {"value": statistics.median(rates), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"median of {samples} runs of {min(steps)}-{max(steps)} decode steps of config 0 (after the "
                      f"prompt forward; runs {', '.join(f'{r:.0f}' for r in rates)} tok/s), {threads}-thread team "
                      f"(one per physical core), {'AVX-512 VNNI' if vnni else 'scalar'} integer dots, "
                      f"{os.cpu_count()} logical CPUs"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    steps = []
    for i in range(args.warmup + args.steps):
        b = cpu_baseline(args.cpu_seconds)
        if i >= args.warmup:
            steps.append(b["value"])
    v = statistics.median(steps)
    b["value"] = v
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * STEPS_PER_GEN / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int16xint4->int32",
            "data": "synthetic", "config": config_dict(args),
            "cpu_baseline": b, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


SWEEP_SHAPES = [(2304, 768), (768, 768), (3072, 768), (768, 3072), (50257, 768)]  # (out, in)
SWEEP_AFFINE = ["int8-g32", "int8-g64", "int8-g128", "int8-ch", "int4-g32", "int4-g64", "int4-g128", "int4-ch"]


PREFILL_T = 476
PREFILL_FORMATS = ["int8-ch-a16", "int4-g32-a16"]
PREFILL_INT_OPS = 2 * PREFILL_T * LAYER_WEIGHTS  # 80.86 G int-ops of the layer GEMMs (head: last token only)


def run_prefill(args):
    """Config 2: 476 ids ~ U[0, 50257) (seed 2), batch 1, one forward of the
    whole prompt (embedding, 12 layers of prefill GEMMs and attention, the
    last token's head + argmax), L2 flushed before each step. Device time by
    CUDA events around llmq_model_forward on the library's stream (the call
    copies the 1.9 KB of ids in and the argmax out); one JSON line per format."""
    import torch

    from llm_mojo_b200 import build, synth
    from llm_mojo_b200.model import Model
    from llm_mojo_b200.tensor import Context

    build.build()
    torch.cuda.set_device(0)
    ctx = Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    tensors = synth.gpt2_random_init(0)
    ids = synth.uniform_ids(PREFILL_T, 2)
    for fmt in PREFILL_FORMATS:
        model = Model(ctx, tensors, dtype=fmt)
        times, walls = [], []
        with torch.cuda.stream(stream):
            for i in range(args.warmup + args.steps):
                flush.zero_()
                s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record(stream)
                t0 = time.perf_counter()
                model.forward(ids, 0)
                walls.append(time.perf_counter() - t0)
                e0.record(stream)
                if i >= args.warmup:
                    times.append((s0, e0))
            stream.synchronize()
        ms = statistics.median(s0.elapsed_time(e0) for s0, e0 in times)
        wall = statistics.median(walls[args.warmup:])
        print(json.dumps({"workload": "config 2 prefill", "format": fmt, "tokens": PREFILL_T,
                          "ms_per_prompt": round(ms, 4), "prefill_tok_s": round(PREFILL_T / (ms / 1000.0), 1),
                          "e2e_tok_s": round(PREFILL_T / wall, 1),
                          "layer_int_gops": round(PREFILL_INT_OPS / (ms / 1000.0) / 1e9, 1),
                          "l2": "flushed before each step", "steps": args.steps, "warmup": args.warmup}))
        model.free()
    ctx.close()
    return 0


BATCH_SEQS, BATCH_PROMPT, BATCH_STEPS = 256, 128, 128


def cpu_batched_baseline(seconds: float):
    """The CPU oracle on config 3's first sequence: its 128-token prompt and
    as many greedy tokens as fit in `seconds`; returns generated tok/s of a
    whole sequence (prompt time + 128 x the mean decode-step time), the rate
    of the reference, which decodes sequences one after another."""
    from llm_mojo_b200 import synth
    from oracle import oracle as O

    t = synth.gpt2_random_init(0)
    m = O.Model(t, max_t=BATCH_PROMPT + BATCH_STEPS)
    prompt = synth.uniform_ids(BATCH_SEQS * BATCH_PROMPT, 3).reshape(BATCH_SEQS, BATCH_PROMPT)[0]
    t0 = time.perf_counter()
    logits = m.forward(prompt, 0)
    t_prompt = time.perf_counter() - t0
    n, pos, t1 = 0, BATCH_PROMPT, time.perf_counter()
    while n < BATCH_STEPS - 1 and (n == 0 or time.perf_counter() - t1 < seconds):
        nxt = int(O.lib().oq_argmax(O.ptr(logits), m.V))
        logits = m.forward([nxt], pos)
        pos += 1
        n += 1
    t_step = (time.perf_counter() - t1) / n
    m.close()
    per_seq = t_prompt + (BATCH_STEPS - 1) * t_step
    threads = int(O.lib().oq_threads())
    return {"value": BATCH_STEPS / per_seq, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"sequence 0 of config 3: its prompt forward ({t_prompt:.2f} s) and {n} decode steps "
                      f"({t_step * 1000:.1f} ms each), extrapolated to its 128 tokens; sequences run one after "
                      f"another; {threads}-thread team"}


def run_batched(args):
    """Config 3: 256 independent sequences, each a 128-token prompt ~ U[0, V)
    (seed 3) then 128 greedy tokens, int4-g32-a16 + int8 head + int8 KV.
    Sequences are split evenly across the ranks (strong scaling); after its
    generation every rank joins one NCCL all-gather of the ids. value: all
    ranks' generated tokens / the max over ranks of the device time of one
    whole generation (prompts and ids in HBM, the gather included)."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from llm_mojo_b200 import build, synth
    from llm_mojo_b200.model import Batch, Model
    from llm_mojo_b200.tensor import Context

    from llm_mojo_b200.shard import gather_blocks, shard_range

    build.build()
    n_seqs, n_steps = args.batch_seqs, args.batch_steps
    b_lo, b_hi = shard_range(n_seqs, world, rank)
    per = b_hi - b_lo
    ctx = Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    model = Model(ctx, synth.gpt2_random_init(0), max_t=BATCH_PROMPT + n_steps)
    batch = Batch(model, per, BATCH_PROMPT)
    prompts = synth.uniform_ids(BATCH_SEQS * BATCH_PROMPT, 3).reshape(BATCH_SEQS, BATCH_PROMPT)
    mine = np.ascontiguousarray(prompts[b_lo:b_hi])
    prompts_dev = torch.from_numpy(mine).cuda()
    ids_dev = torch.zeros((per, n_steps), dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def gather():
        return gather_blocks(ids_dev, world)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    times = []
    with torch.cuda.stream(stream):
        for i in range(args.warmup + args.steps):
            flush.zero_()
            barrier()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            batch.generate_async(prompts_dev, n_steps, ids_dev)
            gather()
            e0.record(stream)
            barrier()
            if i >= args.warmup:
                times.append(s0.elapsed_time(e0))
    ms = torch.tensor([statistics.mean(times)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    # e2e: host prompts and host ids through llmq_batch_generate, then the gather
    e2e = []
    for i in range(2):
        barrier()
        t0 = time.perf_counter()
        ids = batch.generate(mine, n_steps)
        ids_dev.copy_(torch.from_numpy(ids))
        host_ids = gather().cpu()
        barrier()
        e2e.append(time.perf_counter() - t0)
    e2e_s = torch.tensor([min(e2e)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_s.item())
    total = n_seqs * n_steps
    if rank == 0:
        check_ids = host_ids.reshape(n_seqs, n_steps).numpy()
        single = model.generate(list(prompts[n_seqs - 1]), n_steps)
        cpu = None if args.no_cpu_baseline else cpu_batched_baseline(min(args.cpu_seconds, 15.0))
        line = {"metric": "int4-g32-a16 batched decode tok/s (b=256/box)", "value": total / (ms / 1000.0),
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int16xint4->int32",
                "data": "synthetic",
                "config": {"workload": "config 3: 256 sequences x (128-token prompt ~ U[0, 50257) seed 3 + 128 "
                                       "greedy tokens), GPT-2 124M int4-g32-a16 + int8-ch head + int8 KV, "
                                       "random-init weights (seed 0)",
                           "global_batch": n_seqs, "seq_len": BATCH_PROMPT + n_steps,
                           "parallelism": f"sequences split over {world} ranks, one NCCL all-gather of the ids",
                           "l2": "flushed between steps (256 MiB write)"},
                "e2e": {"value": total / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": per * BATCH_PROMPT * 4,
                        "d2h_bytes_per_step": n_seqs * n_steps * 4},
                "last_sequence_matches_single_decode": bool(list(check_ids[-1]) == list(single)),
                # per generation: the prompt (embed, 12 x (2 LayerNorm + 4 x (split + GEMM) + store +
                # attention), gather, head GEMM (quantizing inside), argmax, state) and 127 decode-step
                # graphs (advance, embed, 12 x (3 GEMMs quantizing inside + quantize + GEMM for the
                # 3072-column rows + attention), head GEMM, argmax)
                "gpu_launches": args.steps * ((1 + 12 * 12 + 1 + 1 + 1 + 1) + (n_steps - 1) * (2 + 12 * 6 + 2)),
                "cpu_baseline": cpu}
        print(json.dumps(line))
    batch.free()
    model.free()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def batched_sub(model, stream, flush, world, rank, reps=2, warmup=1):
    """Config 3 inside the default bench line: 256 sequences x (128-token
    prompt ~ U[0, V) seed 3 + 128 greedy tokens) split evenly over the ranks
    (strong scaling), then one NCCL all-gather of the ids, on the config-0
    model's weights. Device time by CUDA events around one whole generation
    (prompts and ids in HBM, the gather included), L2 flushed before each;
    the max over ranks of the mean of `reps` timed generations."""
    import torch
    import torch.distributed as dist

    from llm_mojo_b200 import synth
    from llm_mojo_b200.model import Batch
    from llm_mojo_b200.shard import gather_blocks, shard_range

    b_lo, b_hi = shard_range(BATCH_SEQS, world, rank)
    per = b_hi - b_lo
    batch = Batch(model, per, BATCH_PROMPT)
    prompts = synth.uniform_ids(BATCH_SEQS * BATCH_PROMPT, 3).reshape(BATCH_SEQS, BATCH_PROMPT)
    prompts_dev = torch.from_numpy(np.ascontiguousarray(prompts[b_lo:b_hi])).cuda()
    ids_dev = torch.zeros((per, BATCH_STEPS), dtype=torch.int32, device="cuda")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + reps):
            flush.zero_()
            barrier()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            batch.generate_async(prompts_dev, BATCH_STEPS, ids_dev)
            all_ids = gather_blocks(ids_dev, world)
            e0.record(stream)
            barrier()
            if i >= warmup:
                times.append(s0.elapsed_time(e0))
    ms = torch.tensor([statistics.mean(times)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    head = [int(v) for v in all_ids.reshape(BATCH_SEQS, BATCH_STEPS)[-1, :4].cpu()]
    batch.free()
    return {"metric": "int4-g32-a16 batched decode tok/s (b=256/box)",
            "value": BATCH_SEQS * BATCH_STEPS / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
            "scaling": "strong", "seqs": BATCH_SEQS, "prompt_len": BATCH_PROMPT, "gen_tokens": BATCH_STEPS,
            "ms_per_generation": ms, "steps": reps, "warmup": warmup,
            "parallelism": f"sequences split over {world} ranks, one NCCL all-gather of the ids",
            "workload": "config 3: 256 sequences x (128-token prompt ~ U[0, 50257) seed 3 + 128 greedy tokens), "
                        "GPT-2 124M int4-g32-a16 + int8-ch head + int8 KV, random-init weights (seed 0)",
            "l2": "flushed between generations (256 MiB write)", "last_seq_ids_head": head}


PPL_IDS, PPL_SEED = 65536, 4


def cpu_ppl_baseline(seconds: float):
    """The CPU oracle on config 4's first window, int4-g32-a16, cut to the
    tokens it forwards in about `seconds` (from 64 up, doubling): windows/s
    extrapolated linearly to the 1024-token window (optimistic: attention
    grows faster), with its rows scored."""
    from llm_mojo_b200 import synth
    from oracle import oracle as O

    t = synth.gpt2_random_init(0)
    ids = synth.zipf_ids(PPL_IDS, PPL_SEED)
    m = O.Model(t)
    n, dt = 64, 0.0
    while True:
        t0 = time.perf_counter()
        lm = m.forward_all(ids[:n])
        st = np.zeros((6, n - 1))
        targets = np.ascontiguousarray(ids[1:n + 1], dtype=np.int32)
        O.lib().oq_score_rows(O.ptr(np.ascontiguousarray(lm)), None, O.ptr(targets), lm.shape[1], 0, n - 1,
                              O.ptr(st), n - 1)
        dt = time.perf_counter() - t0
        if dt * 2 > seconds or n >= 1024:
            break
        n *= 2
    m.close()
    threads = int(O.lib().oq_threads())
    return {"value": 1.0 / (dt * 1024 / n), "unit": "windows/s", "cores": threads, "kind": "port",
            "sample": f"int4-g32-a16 forward_all + score_rows of the first {n} tokens of window 0 in {dt:.2f} s, "
                      f"extrapolated linearly to 1024 tokens; one format, no float32 base; {threads}-thread team"}


def run_ppl(args):
    """Config 4: 65,536 ids ~ Zipf(1.1) over the vocabulary (seed 4), windows
    of 1024 every 512 (127 windows, every token after the first scored once),
    formats f32, bf16, int4-g32-a16 and GGUF Q4_K (Q6_K head), each against
    float32 on the same windows. Windows split round-robin over the ranks;
    the totals meet in one all-reduce. value: windows / the max over ranks of
    the device time of all of them (the four formats and the f32 base)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    from llm_mojo_b200 import build, synth
    from llm_mojo_b200.evaluate import Harness, rank_windows, schedule
    from llm_mojo_b200.model import FloatModel, Model
    from llm_mojo_b200.tensor import Context

    build.build()
    ctx = Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    tensors = synth.gpt2_random_init(0)
    base = FloatModel(ctx, tensors, "f32")
    models = {"f32": base, "bf16": FloatModel(ctx, tensors, "bf16"), "int4-g32-a16": Model(ctx, tensors),
              "gguf-q4_k": FloatModel(ctx, tensors, "gguf-q4_k")}
    ids = synth.zipf_ids(PPL_IDS, PPL_SEED)
    wins = schedule(len(ids))
    mine = rank_windows(wins, world, rank)
    with torch.cuda.stream(stream):
        warm = Harness(ctx, models, base)
        for w in mine[:1]:
            warm.score_window(ids, *w)
        del warm
        h = Harness(ctx, models, base)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        t0 = time.perf_counter()
        for w in mine:
            h.score_window(ids, *w)
        e0.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ms = torch.tensor([s0.elapsed_time(e0), wall * 1000.0], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        h.reduce(world)
    rep = h.report()
    if rank == 0:
        ms_dev, ms_wall = float(ms[0]), float(ms[1])
        cpu = None if args.no_cpu_baseline else cpu_ppl_baseline(min(args.cpu_seconds, 20.0))
        line = {"metric": "perplexity windows/s (4 formats vs f32, 1024-token windows)",
                "value": len(wins) / (ms_dev / 1000.0), "unit": "windows/s", "n_gpus": world, "steps": 1,
                "warmup": 1, "ms_per_step": ms_dev / max(1, len(mine)), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32/bf16/int16xint4/gguf",
                "data": "synthetic",
                "config": {"workload": "config 4: 65,536 ids ~ Zipf(1.1) seed 4, window 1024 stride 512, 127 windows; "
                                       "GPT-2 124M random-init (seed 0) in f32, bf16, int4-g32-a16, GGUF Q4_K "
                                       "(Q6_K head), each vs f32",
                           "global_batch": len(wins), "seq_len": WINDOW_T,
                           "parallelism": f"windows round-robin over {world} ranks, one all-reduce of the totals"},
                "e2e": {"value": len(wins) / (ms_wall / 1000.0), "unit": "windows/s",
                        "h2d_bytes_per_step": 4 * 1024 * 4, "d2h_bytes_per_step": 0},
                "formats": rep, "gpu_launches": None, "cpu_baseline": cpu}
        print(json.dumps(line))
    for m in models.values():
        m.free()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


WINDOW_T = 1024


ROTATE_BYTES = int(2.2 * 126e6)  # the rotation's copies together: over twice B200's L2


def clone(w, make):
    """Another device copy of w from the host arrays it was made from."""
    from llm_mojo_b200.tensor import GGUFMatrix, QuantMatrix
    if isinstance(w, QuantMatrix):
        return QuantMatrix(w.ctx, w.bits, w.group_param, w.sym, w.a16, w.rows, w.cols, w.codes, w.scale, w.zp)
    if isinstance(w, GGUFMatrix):
        return GGUFMatrix(w.ctx, w.kind, w.blocks, w.rows, w.cols)
    return make()


def run_sweep(args):
    """Config 1: x ~ N(0,1) (seed 1), W ~ N(0, 0.02) quantized per format;
    GB/s of packed weight bytes per one-token GEMV.

    Primary figure ("us", "GB/s"): R copies of the weight, together more
    than 2.2x the 126 MB L2, launched back to back as one CUDA graph (one
    launch per copy, so every launch reads its weight from HBM and no launch
    waits on a flush); per-launch time = graph replay time / R, median over
    args.steps replays. Secondary ("us_flushed"): one launch right after a
    256 MiB L2-flushing write, median of args.steps launches; below ~10 us it
    measures the launch-after-flush floor, not bandwidth."""
    import ctypes as C

    import torch

    from llm_mojo_b200 import build
    from llm_mojo_b200 import gguf_blocks as G
    from llm_mojo_b200._lib import BIAS, check, lib
    from llm_mojo_b200.tensor import Context, DenseMatrix, GGUFMatrix, QuantMatrix, parse_dtype

    build.build()
    torch.cuda.set_device(0)
    ctx = Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    peak, peak_kind = peaks()
    rng = np.random.default_rng(1)
    only_fmt, only_shape = None, None
    if args.sweep_only:
        only_fmt, _, shp = args.sweep_only.partition(":")
        only_shape = tuple(int(v) for v in shp.split("x")) if shp else None
    for out_, in_ in SWEEP_SHAPES:
        x_host = rng.standard_normal(in_).astype(np.float32)  # drawn for every shape: filters keep the inputs
        if only_shape and (out_, in_) != only_shape:
            continue
        src = (np.random.default_rng(out_ * 7 + in_).standard_normal((in_, out_), dtype=np.float32) *
               np.float32(0.02)).astype(np.float32)  # [IN, OUT] (Hugging Face layout)
        x = torch.from_numpy(x_host).cuda()
        b = torch.zeros(out_, dtype=torch.float32, device="cuda")
        y = torch.zeros(out_, dtype=torch.float32, device="cuda")
        cases = []
        for f in SWEEP_AFFINE:
            bits, group, sym, _ = parse_dtype(f)
            cases.append((f + "-a16", lambda bits=bits, group=group, sym=sym:
                          QuantMatrix.from_f32(ctx, src, bits, group, sym, True, True)))
            cases.append((f, lambda bits=bits, group=group, sym=sym:
                          QuantMatrix.from_f32(ctx, src, bits, group, sym, False, True)))
        for t in (G.Q4_0, G.Q4_1, G.Q8_0, G.Q4_K, G.Q5_K, G.Q6_K):
            cases.append((G.NAMES[t], lambda t=t: GGUFMatrix(ctx, t, G.quantize(np.ascontiguousarray(src.T), t),
                                                            out_, in_)))
        for dt in ("f32", "f16", "bf16"):
            # layer matrices stay [IN, OUT]; the head is wte [V, C]
            cases.append((dt, lambda dt=dt: DenseMatrix(ctx, dt, src if out_ != 50257 else np.ascontiguousarray(src.T))))
        for name, make in cases:
            if only_fmt and name != only_fmt:
                continue
            try:
                w = make()
            except Exception as e:  # a format the shape does not divide into
                print(json.dumps({"workload": "config 1 GEMV sweep", "format": name, "shape": [out_, in_],
                                  "skipped": str(e)[:80]}))
                continue
            is_head = out_ == 50257
            def launch(w):
                if is_head:
                    check(lib().llmq_head(ctx.h, w.h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 1, in_,
                                          out_), ctx.h)
                else:
                    check(lib().llmq_linear(ctx.h, w.h, C.c_void_p(x.data_ptr()), C.c_void_p(b.data_ptr()),
                                            C.c_void_p(y.data_ptr()), 1, in_, out_, BIAS), ctx.h)
            times = []
            with torch.cuda.stream(stream):
                for i in range(args.warmup + args.steps):
                    flush.zero_()
                    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s0.record(stream)
                    launch(w)
                    e0.record(stream)
                    if i >= args.warmup:
                        times.append((s0, e0))
                stream.synchronize()
            ms_flushed = statistics.median(s0.elapsed_time(e0) for s0, e0 in times)
            nbytes = w.nbytes()
            # rotation: R copies over 2.2x L2, one graph of R back-to-back launches
            reps = max(2, -(-ROTATE_BYTES // nbytes))
            copies = [w] + [clone(w, make) for _ in range(reps - 1)]
            with torch.cuda.stream(stream):
                for wc in copies:  # eager once: any lazily made per-weight state exists before capture
                    launch(wc)
            stream.synchronize()
            graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
            ctx.set_stream(cap.cuda_stream)
            try:
                with torch.cuda.graph(graph, stream=cap):
                    for wc in copies:
                        launch(wc)
            finally:
                ctx.set_stream(stream.cuda_stream)
            gtimes = []
            with torch.cuda.stream(stream):
                for i in range(args.warmup + args.steps):
                    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s0.record(stream)
                    graph.replay()
                    e0.record(stream)
                    if i >= args.warmup:
                        gtimes.append((s0, e0))
                stream.synchronize()
            ms = statistics.median(s0.elapsed_time(e0) for s0, e0 in gtimes) / reps
            del graph
            gbs = nbytes / (ms / 1000.0) / 1e9
            print(json.dumps({"workload": "config 1 GEMV sweep", "format": name, "shape": [out_, in_],
                              "weight_bytes": nbytes, "us": round(ms * 1000, 2), "GB/s": round(gbs, 1),
                              "frac_of_hbm": round(gbs / peak, 4), "peak_kind": peak_kind,
                              "copies": reps, "l2": f"rotation over {reps} copies ({reps * nbytes >> 20} MiB), "
                                                    "one graph of back-to-back launches",
                              "us_flushed": round(ms_flushed * 1000, 2),
                              "GB/s_flushed": round(nbytes / (ms_flushed / 1000.0) / 1e9, 1)}))
            for wc in copies:
                wc.free()
    ctx.close()
    return 0


def config_dict(args):
    return {"workload": "config 0: GPT-2 124M batch-1 greedy decode, int4-g32-a16 layers + int8-ch head + "
                        "int8 KV, prompt [50256] then 100 tokens, random-init weights (seed 0)",
            "global_batch": args.gpus, "seq_len": 101, "parallelism": f"replicas{args.gpus}",
            "l2": "flushed between steps (256 MiB write)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "sweep", "prefill", "batched", "ppl"],
                    help="decode: config 0 (the default bench line); sweep: config 1, the one-token GEMV of every "
                         "format at every shape, one JSON line each; prefill: config 2, one line per format; "
                         "batched: config 3, sequences split over the ranks; ppl: config 4, windows split over "
                         "the ranks")
    ap.add_argument("--batch-seqs", type=int, default=256,
                    help="batched workload: sequences (config 3 has 256; fewer for profiling captures)")
    ap.add_argument("--batch-steps", type=int, default=128,
                    help="batched workload: greedy tokens per sequence (config 3 has 128)")
    ap.add_argument("--sweep-only", default=None, metavar="FORMAT[:OUTxIN]",
                    help="sweep workload: time only this format (e.g. int8-ch-a16), optionally at one shape "
                         "(e.g. int8-ch-a16:50257x768), for profiling captures")
    ap.add_argument("--no-batched", action="store_true",
                    help="leave out the config-3 batched decode sub-object of the default line")
    ap.add_argument("--mode", default=None, choices=["cluster", "persistent", "graph", "eager"],
                    help="decode mode of the config-0 model (default: the library's default for its formats)")
    ap.add_argument("--profile", action="store_true",
                    help="after the timed region, run one generation with the persistent kernel's per-phase "
                         "timers and print them (microseconds per token) to stderr")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "sweep":
        return run_sweep(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "batched":
        return run_batched(args)
    if args.workload == "ppl":
        return run_ppl(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    from llm_mojo_b200 import build, synth
    from llm_mojo_b200._lib import check, lib
    from llm_mojo_b200.model import Model
    from llm_mojo_b200.tensor import Context

    build.build()
    ctx = Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    model = Model(ctx, synth.gpt2_random_init(0))
    if args.mode:
        model.set_mode(args.mode)
    prompt_dev = torch.tensor(PROMPT, dtype=torch.int32, device="cuda")
    ids_dev = torch.zeros(STEPS_PER_GEN, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    import ctypes as C

    def gen_async():
        check(lib().llmq_generate_async(ctx.h, model.h, C.c_void_p(prompt_dev.data_ptr()), len(PROMPT),
                                        STEPS_PER_GEN, C.c_void_p(ids_dev.data_ptr())), ctx.h)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            gen_async()
            flush.zero_()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with Clocks(local) as clk:
            for s, e in evs:
                s.record(stream)
                gen_async()
                e.record(stream)
                flush.zero_()
            stream.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        step_ms = [s.elapsed_time(e) for s, e in evs]
        total_ms = sum(step_ms)
        ids = ids_dev.cpu().numpy().copy()

        # e2e: the public host-buffer call, copies inside the timed region.
        e2e_ms = []
        for _ in range(max(3, args.steps // 2)):
            flush.zero_()
            stream.synchronize()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            out = model.generate(PROMPT, STEPS_PER_GEN)
            e0.record(stream)
            stream.synchronize()
            e2e_ms.append(s0.elapsed_time(e0))
        assert list(out) == list(ids)

    batched = None if args.no_batched else batched_sub(model, stream, flush, world, rank)

    if args.profile:
        model.profile(True)
        model.generate(PROMPT, STEPS_PER_GEN)
        mhz = torch.cuda.get_device_properties(local).clock_rate / 1000.0 if hasattr(
            torch.cuda.get_device_properties(local), "clock_rate") else 1965.0
        for i, d in enumerate(model.profile_read()):
            steps = max(1, d.pop("steps"))
            us = {k: v / steps / mhz for k, v in d.items()}
            tot = sum(v for k, v in us.items() if k != "ring waits" and not k.startswith("in: "))
            print(f"[profile] CTA {'0' if i == 0 else 'grid/2'}: {tot:.1f} us/token at {mhz:.0f} MHz: " +
                  ", ".join(f"{k} {v:.2f}" for k, v in us.items()), file=sys.stderr)
        model.profile(False)

    t_max = total_ms
    e2e_avg = statistics.mean(e2e_ms)
    if world > 1:
        tt = torch.tensor([total_ms, e2e_avg], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, e2e_avg = float(tt[0]), float(tt[1])
        all_ids = [torch.zeros(STEPS_PER_GEN, dtype=torch.int32, device="cuda") for _ in range(world)]
        dist.all_gather(all_ids, ids_dev)
    tokens = world * args.steps * STEPS_PER_GEN
    value = tokens / (t_max / 1000.0)
    peak, peak_kind = peaks()
    # roofline: the step is one launch of the persistent decode kernel (the
    # dominant, and only, kernel of the timed region); its algorithmic bytes
    # are the weights of every token plus the KV cache each token reads.
    kv_bytes = 19584 * sum(p + 1 for p in range(STEPS_PER_GEN))
    launch_bytes = STEPS_PER_GEN * TOKEN_BYTES + kv_bytes
    launch_ms = total_ms / args.steps
    achieved = launch_bytes / (launch_ms / 1000.0) / 1e9
    if rank == 0:
        cpu = None if args.no_cpu_baseline else cpu_baseline(args.cpu_seconds)
        launches_per_token = model.n_layer * 5 + 2
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16xint4->int32", "data": "synthetic", "config": config_dict(args),
            "e2e": {"value": world * STEPS_PER_GEN / (e2e_avg / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * len(PROMPT), "d2h_bytes_per_step": 4 * STEPS_PER_GEN},
            "roofline": {"bound": "hbm", "kernel": ("cluster_decode_kernel" if model.mode() == "cluster" else
                                                     "mega_decode_kernel") + " (one launch = the 100-token generation)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": MEGA_TRAFFIC_BYTES if model.mode() == "persistent" else None,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                           "(profiles/mega_decode_kernel.txt)",
                         "algorithmic_bytes_per_launch": launch_bytes, "avg_launch_ms": launch_ms},
            "weight_bytes_per_token": TOKEN_BYTES,
            "effective_weight_gbs": TOKEN_BYTES * STEPS_PER_GEN * args.steps / (total_ms / 1000.0) / 1e9,
            "gpu_launches": args.steps * (1 if model.mode() in ("persistent", "cluster") else
                                          1 + STEPS_PER_GEN * launches_per_token),
            "decode_mode": model.mode(),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "ids_head": [int(i) for i in ids[:8]],
            "batched": batched,
        }
        print(json.dumps(line))
    model.free()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
