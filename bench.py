#!/usr/bin/env python
"""GRPO RL steps/sec (+ rollout decode tok/s) on the Qwen3-VL-4B architecture, 1..8 B200s.

Workload (random-init weights, synthetic data): groups_per_batch 8 x group_size 8
= 64 sequences per RL step, one 448x448 uniform-random RGB image (784 patches ->
196 image tokens) + 64 uniform-random prompt tokens per prompt, 128 sampled
tokens (temperature 0.7, top-p 0.9, top-k 5), geodesic reward on coordinates
parsed from the response (0 when unparseable), PPO clip 0.2, KL to a frozen
reference copy of the initial weights, AdamW lr 5e-7, 2 minibatches, bf16
compute with fp32 master weights and moments.  One RL step = vision encode ->
prefill -> 128-token KV-cache decode -> rewards -> reference + old-policy scoring
-> 2 x (forward, backward, AdamW).  With N GPUs the global batch stays 64
(strong scaling): each rank rolls out 8/N groups, FSDP shards the optimizer state.

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
synchronize and timed with CUDA events on the launching stream; the max over
ranks is reported.  The per-step working set (8.8 GB of weights) exceeds the
126 MB L2, so no flush is needed.  ``e2e`` re-times K steps by wall clock
through the public ``GRPOTrainer.step`` API, which copies the step's images
from pinned host memory and reads back tokens, rewards and metrics.
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

METRIC = "GRPO RL steps/sec + rollout decode tok/s, Qwen3-VL-4B, 1/2/4/8 B200"

# Named workloads.  grpo_4b is the headline configuration; the others are the companion workloads
# (tiny smoke run, two-image True/False with short answers, 8B with long answers).
WORKLOADS = {
    "grpo_4b": dict(preset="qwen3vl_4b", env="synthetic_geo", groups=8, group_size=8, image=448, prompt_tokens=64,
                    max_new=128, minibatches=2),
    "tiny": dict(preset="tiny", env="synthetic_parity", groups=4, group_size=4, image=64, prompt_tokens=16,
                 max_new=16, minibatches=1),
    "truefalse_4b": dict(preset="qwen3vl_4b", env="synthetic_truefalse", groups=32, group_size=8, image=384,
                         prompt_tokens=48, max_new=8, minibatches=2),
    # rollout only (inference): batch 64, one 448x448 image + 64 prompt tokens, 128 new tokens; the value is
    # generated tokens per second of the whole rollout (vision + prefill + decode), DP over ranks by default
    "rollout_4b": dict(preset="qwen3vl_4b", env="synthetic_geo", groups=8, group_size=8, image=448, prompt_tokens=64,
                       max_new=128, minibatches=1, mode="rollout"),
    # 8B: FSDP over all ranks for the update, rollout tensor parallel over pairs of GPUs (TP-2 x DP-N/2)
    "grpo_8b": dict(preset="qwen3vl_8b", env="synthetic_geo", groups=16, group_size=8, image=672, prompt_tokens=128,
                    max_new=512, minibatches=2, rollout="tp", tp_size=2),
}



def _data_desc(args) -> str:
    """What the synthetic inputs of the workload are (the JSON line's ``data`` field)."""
    n_img = 2 if args.env == "synthetic_truefalse" else 1
    targets = {"synthetic_geo": "uniform-on-sphere lat/lon targets",
               "synthetic_truefalse": "Bernoulli(0.5) True/False labels",
               "synthetic_parity": "parity-of-first-token reward"}.get(args.env, args.env)
    return (f"synthetic ({n_img} uniform-random {args.image}x{args.image} RGB image{'s' if n_img > 1 else ''} and "
            f"{args.prompt_tokens} uniform-random prompt ids per prompt, {targets}), random-init weights")

def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="grpo_4b",
                    help="named workload; its fields are the defaults of the flags below")
    ap.add_argument("--preset", default=None)
    ap.add_argument("--groups", type=int, default=None)
    ap.add_argument("--group-size", type=int, default=None)
    ap.add_argument("--max-new", type=int, default=None)
    ap.add_argument("--prompt-tokens", type=int, default=None)
    ap.add_argument("--image", type=int, default=None)
    ap.add_argument("--minibatches", type=int, default=None)
    ap.add_argument("--top-k", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--fsdp-params", choices=["gathered", "sharded"], default="gathered",
                    help="gathered: bf16 parameters stay all-gathered (pushed by the fused AdamW); sharded: "
                         "decoder-layer weights are all-gathered inside the GEMMs that consume them")
    ap.add_argument("--rollout", choices=["tp", "dp"], default=None,
                    help="N>1: tensor-parallel decode (tp) or each rank decodes its own groups (dp, the default)")
    ap.add_argument("--tp-size", type=int, default=None,
                    help="GPUs per tensor-parallel rollout group with --rollout tp (default: all)")
    args = ap.parse_args()
    args.mode = WORKLOADS[args.workload].get("mode", "train")
    for k, v in WORKLOADS[args.workload].items():
        if getattr(args, k, None) is None:
            setattr(args, k, v)
    if args.rollout is None:
        args.rollout = "dp"
    if args.tp_size is None:
        args.tp_size = 0
    return args


def reference_arm(args):
    why = ("reference is JAX 0.6.1/Flax/Optax (uv.lock); no jax, flax or optax wheel exists in the offline "
           "wheelhouse, so `pip install --no-deps` of the package succeeds but it cannot be imported")
    print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": why, "n_gpus": args.gpus}))
    return 0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1])]
        pw = [num(r[3]) or 0.0 for r in rows]
        loaded = [num(r[1]) for r in rows if (num(r[3]) or 0) > 300 and num(r[1])] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": num(rows[0][2]),
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from vlmrl import ops
    from vlmrl.core.optim import AdamWConfig
    from vlmrl.core.ppo import TrainerConfig
    from vlmrl.core.trainer import GRPOTrainer
    from vlmrl.envs.base import create_env
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.utils.tokenizer import ByteTokenizer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    spec = get_preset(args.preset)
    merge_px = spec.vision.patch_size * spec.vision.spatial_merge_size
    image_tokens = (args.image // merge_px) ** 2
    tok = ByteTokenizer(spec.text.vocab_size)
    cfg = TrainerConfig(temperature=0.7, top_p=0.9, top_k=args.top_k, max_new_tokens=args.max_new,
                        groups_per_batch=args.groups, group_size=args.group_size, kl_ref_coef=0.01,
                        n_minibatches=args.minibatches, clip_epsilon=0.2, adaptive_kl=False)
    adamw = AdamWConfig(lr=5e-7, weight_decay=0.01, max_grad_norm=1.0)
    env = create_env(args.env, tok, image_size=args.image, prompt_tokens=args.prompt_tokens, num_tasks=1024, seed=0)
    if world > 1:
        from vlmrl.parallel.fsdp import build_fsdp_models

        model, ref_model, train_state = build_fsdp_models(spec, adamw, seed=0, device=dev,
                                                          shard_params=args.fsdp_params == "sharded")
    else:
        model = Qwen3VLModel(spec, device=dev, dtype=torch.bfloat16, seed=0)
        text_units = {k: v for k, v in model.params.units.items() if k != "visual"}
        ref_model = Qwen3VLModel(spec, units=text_units, device=dev, dtype=torch.bfloat16)
        train_state = None
    trainer = GRPOTrainer(model, tok, env, cfg, adamw, ref_model=ref_model, seed=0, rank=rank, world_size=world,
                          train_state=train_state,
                          tp_rollout=(world > 1 and args.rollout == "tp"),
                          tp_size=min(args.tp_size, world) if args.tp_size else 0)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rollout_only = args.mode == "rollout"
    run = trainer.rollout if rollout_only else trainer.step
    for _ in range(args.warmup):
        run()
    ops.check_errors()

    # ---- device-timed region
    barrier()
    torch.cuda.synchronize()
    gen = trainer.generator
    l0, g0 = ops.launch_count(), gen.graph_kernel_launches
    decode_ms, decode_tokens, gen_tokens = 0.0, 0, 0
    with ClockSampler(dev.index) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        metrics = []
        for _ in range(args.steps):
            m = run()
            metrics.append(m)
            decode_ms += gen.decode_time_ms()
            decode_tokens += gen.last_decode_tokens
            gen_tokens += int(m["tokens/generated"])
        end.record()
        torch.cuda.synchronize()
    barrier()
    launches = (ops.launch_count() - l0) + (gen.graph_kernel_launches - g0)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    decode_ms = max_over_ranks(decode_ms / args.steps)
    ops.check_errors()
    clk = clocks.summary()

    # ---- end-to-end (wall clock, public API, includes pinned H2D of images and D2H of results)
    e2e = None
    if not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            run()
        torch.cuda.synchronize()
        barrier()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
        roll_groups = args.groups if trainer.tp is not None else args.groups // world  # rolled out on this rank
        n_img = 2 if args.env == "synthetic_truefalse" else 1
        img_bytes = roll_groups * n_img * args.image * args.image * 3
        prompt_len = n_img * (image_tokens + 2) + args.prompt_tokens
        seqs = args.groups * args.group_size // world                                   # trained on this rank
        # images + prefill ids/positions + packed training ids/positions/indices (int64)
        h2d = img_bytes + roll_groups * prompt_len * 8 * 5
        if not rollout_only:
            h2d += seqs * (prompt_len + args.max_new) * 8 * 5
        d2h = seqs * args.max_new * 12 + 8 * 64                         # tokens, logprobs, lengths, metrics
        if rollout_only:
            e2e = {"value": args.groups * args.group_size * args.max_new / e2e_s, "unit": "generated tokens/s",
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3}
        else:
            e2e = {"value": 1.0 / e2e_s, "unit": "RL steps/s", "h2d_bytes_per_step": int(h2d),
                   "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3}

    total_seqs = args.groups * args.group_size
    decode_tok_s = (total_seqs * (args.max_new - 1)) / (decode_ms / 1e3) if decode_ms > 0 else None
    last = metrics[-1]
    out = {
        "metric": METRIC,
        "value": (total_seqs * args.max_new / (ms / 1e3)) if rollout_only else 1000.0 / ms,
        "unit": "generated tokens/s (rollout)" if rollout_only else "RL steps/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": _data_desc(args),
        "config": {"model": f"{args.preset} architecture (random init)", "global_batch": total_seqs,
                   "seq_len": f"{(2 if args.env == 'synthetic_truefalse' else 1) * (image_tokens + 2) + args.prompt_tokens}"
                              f" prompt + {args.max_new} new",
                   "workload": args.workload,
                   "parallelism": (((f"tp{trainer.tp_size}xdp{world // trainer.tp_size}") if trainer.tp is not None
                                    else f"dp{world}") if rollout_only else
                                   (f"fsdp{world}+tp{trainer.tp_size}x"
                                    f"dp{world // trainer.tp_size}-rollout") if trainer.tp is not None else f"fsdp{world}")
                   + ("-sharded-params" if args.fsdp_params == "sharded" and world > 1 else "")
                   if world > 1 else "single-gpu",
                   "fsdp_comm": getattr(model.params, "comm", None) if world > 1 else None,
                   "groups_per_batch": args.groups, "group_size": args.group_size, "minibatches": args.minibatches,
                   "kl_ref_coef": 0.01, "top_k": args.top_k, "top_p": 0.9, "temperature": 0.7,
                   "kv_cache": ("paged, 64-token blocks, prompt blocks shared per group"
                                if trainer.generator.paged_kv else "contiguous rows"),
                   "l2": "no flush: per-step working set (8.8 GB weights) >> 126 MB L2"},
        "decode_tok_s": decode_tok_s,
        "decode_ms_per_step": decode_ms,
        "rollout_tokens_per_step": gen_tokens / max(1, args.steps),   # already summed over ranks
        "phase_ms": {k: v for k, v in last.items() if k.startswith("time/")},
        "gpu_launches": int(launches),
        "clocks": clk,
        "e2e": e2e,
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        trainer.close()
        close = getattr(model.params, "close", None)
        if close is not None:
            close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
