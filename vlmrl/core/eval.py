"""Sampler benchmark and smoke test (reference ``core/eval.py:1-633``).

``python -m vlmrl.core.eval --ckpt_dir=DIR --prompt "..." [--image img.png]``
samples from a converted checkpoint (or ``--preset`` random weights) and
reports latency and throughput: one untimed warm-up, ``--benchmark_runs``
timed runs (duration mean/std, tokens/s, steady state = runs after the first)
and the first-token latency of a ``max_new_tokens=1`` run, as the reference's
``_benchmark_jax`` does (``core/eval.py:131-206``).  Durations are wall clock
around the public ``sample`` call (which includes the prompt H2D copy and the
token read-back); the device time of the same calls, taken with CUDA events,
is reported next to it.  ``--batch`` replicates the prompt to measure batched
decode throughput.  Launched with ``torchrun --nproc-per-node N`` the batch is split over N processes (one
per GPU, data parallel, NCCL; gloo on CPU): each rank samples its rows with their global row ids, so the
tokens equal a single-process run of the whole batch, and a run's duration is the slowest rank's while its
tokens are summed over ranks.

``--compare_hf`` also times HuggingFace ``generate`` on a local snapshot
(``--hf_model_name`` must be a directory: there is no network), text-only via
``AutoModelForCausalLM`` or with the image via
``Qwen3VLForConditionalGeneration`` (reference ``:209-430``).  The comparison
is written to ``--plot_path`` (a PNG when matplotlib is importable, else the
same data as JSON) and raw metrics to ``--dump_metrics``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from dataclasses import replace
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from vlmrl.core.types import SampleResult, SamplingConfig, VLMInputs


def summaries_from_metrics(metrics: Sequence[Dict[str, float]]) -> Dict[str, float]:
    """Mean/std of duration and throughput; steady state drops the first run (reference ``:74-103``)."""
    if not metrics:
        return {}
    durations = [m["duration"] for m in metrics]
    tokens = [m.get("tokens", 0.0) for m in metrics]
    tps = [(t / d) if d > 0 else 0.0 for t, d in zip(tokens, durations)]
    out = {"runs": len(durations), "duration_mean": statistics.mean(durations),
           "duration_std": statistics.pstdev(durations) if len(durations) > 1 else 0.0,
           "tokens_total": sum(tokens), "throughput_mean": statistics.mean(tps),
           "throughput_std": statistics.pstdev(tps) if len(tps) > 1 else 0.0}
    if len(durations) > 1:
        out["steady_duration_mean"] = statistics.mean(durations[1:])
        out["steady_throughput_mean"] = statistics.mean(tps[1:])
    dev = [m["device_ms"] for m in metrics if m.get("device_ms") is not None]
    if dev:
        out["device_ms_mean"] = statistics.mean(dev)
    return out


def format_summary_table(title: str, summary: Dict[str, float], first_token: Optional[float]) -> str:
    lines = [f"{title}:"]
    if not summary:
        return "\n".join(lines + ["  (no data)"])
    lines.append(f"  runs: {summary['runs']}")
    lines.append(f"  mean duration: {summary['duration_mean']:.3f}s (std {summary['duration_std']:.3f})")
    lines.append(f"  total tokens: {int(summary['tokens_total'])}")
    lines.append(f"  mean throughput: {summary['throughput_mean']:.2f} tok/s (std {summary['throughput_std']:.2f})")
    if "steady_duration_mean" in summary:
        lines.append(f"  steady-state duration: {summary['steady_duration_mean']:.3f}s")
        lines.append(f"  steady-state throughput: {summary['steady_throughput_mean']:.2f} tok/s")
    if "device_ms_mean" in summary:
        lines.append(f"  device time per run: {summary['device_ms_mean']:.2f} ms")
    if first_token is not None:
        lines.append(f"  first-token latency (1 new token run): {first_token:.3f}s")
    return "\n".join(lines)


def _generated_tokens(res: SampleResult) -> int:
    if res.lengths is not None:
        return int(res.lengths.sum())
    return int(res.tokens.numel())


def _dist():
    import torch.distributed as dist

    return dist if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1 else None


def _across_ranks(values: Sequence[float], op: str) -> List[float]:
    """Element-wise max or sum of per-rank values (identity in a single process)."""
    d = _dist()
    if d is None:
        return [float(v) for v in values]
    dev = torch.device("cuda", torch.cuda.current_device()) if d.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=dev)
    d.all_reduce(t, op=d.ReduceOp.MAX if op == "max" else d.ReduceOp.SUM)
    return [float(x) for x in t.cpu()]


def benchmark_native(model, inputs, cfg: SamplingConfig, seed: int, tokenizer, runs: int, row_offset: int = 0
                     ) -> Tuple[SampleResult, Dict[str, float], Optional[float]]:
    """Warm-up + ``runs`` timed calls of the public ``sample``, then a timed 1-token run.  Under data
    parallelism every duration is the slowest rank's and every token count the sum over ranks."""
    from vlmrl.core.sampling import sample
    from vlmrl.utils.rng import RngSeq

    rng = RngSeq(seed)
    cuda = model.device.type == "cuda"
    metrics: List[Dict[str, float]] = []
    last = None
    for i in range(1 + max(1, int(runs))):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) if cuda else None
        if cuda:
            torch.cuda.synchronize()
            ev[0].record()
        t0 = time.perf_counter()
        res = sample(model, None, inputs, cfg, rng.next(), tokenizer=tokenizer, row_offset=row_offset)
        if cuda:
            ev[1].record()
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        last = res
        if i >= 1:
            dev_ms = ev[0].elapsed_time(ev[1]) if cuda else 0.0
            dt, dev_ms = _across_ranks([dt, dev_ms], "max")
            (tokens,) = _across_ranks([_generated_tokens(res)], "sum")
            metrics.append({"duration": dt, "tokens": tokens, "device_ms": dev_ms if cuda else None})
    first = None
    one = replace(cfg, max_new_tokens=1)
    sample(model, None, inputs, one, rng.next(), tokenizer=tokenizer, row_offset=row_offset)
    if cuda:
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    r1 = sample(model, None, inputs, one, rng.next(), tokenizer=tokenizer, row_offset=row_offset)
    if cuda:
        torch.cuda.synchronize()
    (first,) = _across_ranks([time.perf_counter() - t0], "max")
    if r1.tokens.shape[-1] == 0:
        first = None
    return last, summaries_from_metrics(metrics), first


def _hf_dtype(name: str):
    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}.get(name, "auto")


def benchmark_hf(model_dir: str, prompt: str, image: Optional[str], max_new_tokens: int, temperature: float,
                 top_p: float, top_k: Optional[int], runs: int, dtype: str = "auto") -> Dict[str, Any]:
    """Time HuggingFace ``generate`` on a local snapshot (text model, or Qwen3-VL with an image)."""
    import transformers

    if not os.path.isdir(model_dir):
        raise FileNotFoundError(f"--hf_model_name must be a local directory here (no network): {model_dir}")
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    kw = dict(do_sample=temperature > 0, temperature=max(temperature, 1e-5), top_p=top_p, max_new_tokens=max_new_tokens)
    if top_k:
        kw["top_k"] = int(top_k)
    if image:
        from PIL import Image

        proc = transformers.AutoProcessor.from_pretrained(model_dir)
        model = transformers.Qwen3VLForConditionalGeneration.from_pretrained(model_dir, dtype=_hf_dtype(dtype)).to(dev)
        msgs = [{"role": "user", "content": [{"type": "image"}, {"type": "text", "text": prompt}]}]
        text = proc.apply_chat_template(msgs, add_generation_prompt=True)
        enc = proc(text=[text], images=[Image.open(image).convert("RGB")], return_tensors="pt").to(dev)
    else:
        proc = transformers.AutoTokenizer.from_pretrained(model_dir)
        model = transformers.AutoModelForCausalLM.from_pretrained(model_dir, dtype=_hf_dtype(dtype)).to(dev)
        enc = proc([prompt], return_tensors="pt").to(dev)
    n_in = enc["input_ids"].shape[1]
    metrics = []
    out = None
    for i in range(1 + max(1, runs)):
        if dev == "cuda":
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = model.generate(**enc, **kw)
        if dev == "cuda":
            torch.cuda.synchronize()
        if i >= 1:
            metrics.append({"duration": time.perf_counter() - t0, "tokens": float(out.shape[1] - n_in)})
    tok = getattr(proc, "tokenizer", proc)
    return {"summary": summaries_from_metrics(metrics),
            "text": tok.decode(out[0, n_in:], skip_special_tokens=True) if out is not None else ""}


def save_chart(path: str, rows: Dict[str, Dict[str, float]]) -> str:
    """Throughput bar chart (PNG via matplotlib when available, else JSON with the same data)."""
    data = {k: v.get("steady_throughput_mean", v.get("throughput_mean", 0.0)) for k, v in rows.items()}
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    try:
        import matplotlib

        matplotlib.use("Agg")
        import matplotlib.pyplot as plt

        fig, ax = plt.subplots(figsize=(5, 3))
        ax.bar(list(data), list(data.values()))
        ax.set_ylabel("tokens/s")
        fig.tight_layout()
        fig.savefig(path)
        return path
    except Exception:
        alt = os.path.splitext(path)[0] + ".json"
        with open(alt, "w", encoding="utf-8") as fh:
            json.dump(data, fh, indent=2)
        return alt


def build_inputs(model, tokenizer, prompt: str, image: Optional[str], batch: int, pad_id: int):
    """VLMInputs for an image prompt (chat template with the vision block) or a plain token batch."""
    from vlmrl.core.rollout import prepare_prompts

    if image:
        obs = type("Obs", (), {"image": image, "question": prompt})()
        prompts, vision = prepare_prompts(model, tokenizer, [obs] * batch)
        return VLMInputs(prompt_tokens=[p.prompt_tokens for p in prompts], vision=vision,
                         grid_thw=[p.grids for p in prompts], image_pad_id=model.spec.image_token_id)
    ids = np.asarray(tokenizer.encode(prompt, add_special_tokens=False), dtype=np.int64)
    return np.tile(ids[None, :], (batch, 1))


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ckpt_dir", "--model_dir", dest="ckpt_dir", type=str, default="",
                    help="checkpoint directory written by hf_to_jax (the reference README's --model_dir also works)")
    ap.add_argument("--preset", type=str, default="", help="random-init architecture when no checkpoint is given")
    ap.add_argument("--prompt", type=str, default=None)
    ap.add_argument("--image", type=str, default=None)
    ap.add_argument("--max_new_tokens", type=int, default=30)
    ap.add_argument("--temperature", type=float, default=0.1)
    ap.add_argument("--top_p", type=float, default=0.9)
    ap.add_argument("--compat_refeed_last_token", action="store_true",
                    help="start decoding like the reference sampler: drop the prefill logits, decode the last prompt token again")
    ap.add_argument("--top_k", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--pad_id", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1, help="replicate the prompt this many times")
    ap.add_argument("--benchmark_runs", type=int, default=3)
    ap.add_argument("--compare_hf", action="store_true")
    ap.add_argument("--hf_model_name", type=str, default="Qwen/Qwen3-4B")
    ap.add_argument("--hf_dtype", type=str, default="auto")
    ap.add_argument("--plot_path", type=str, default=None)
    ap.add_argument("--dump_metrics", type=str, default=None)
    return ap.parse_args(argv)


def main(argv=None) -> Dict[str, Any]:
    from vlmrl.core.train import load_policy, resolve_pad_and_eos
    from vlmrl.utils.tokenizer import load_tokenizer

    args = parse_args(argv)
    if not args.prompt:
        raise SystemExit("--prompt is required")
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        if not dist.is_initialized():
            dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                    timeout=datetime.timedelta(seconds=300))
        if max(1, args.batch) % world:
            raise SystemExit(f"--batch {args.batch} must be divisible by the {world} processes")
    share = max(1, args.batch) // max(1, world)
    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    model, _ = load_policy(args.ckpt_dir, args.preset, dev, dtype, seed=args.seed)
    tokenizer = load_tokenizer(args.ckpt_dir or None, vocab_size=model.spec.text.vocab_size)
    pad_id, eos_id = resolve_pad_and_eos(tokenizer, model.spec)
    if args.pad_id is not None:
        pad_id = int(args.pad_id)
    cfg = SamplingConfig(temperature=args.temperature, top_p=args.top_p if 0 < args.top_p < 1 else None,
                         top_k=args.top_k, eos_id=eos_id, pad_id=pad_id, max_new_tokens=args.max_new_tokens,
                         compat_refeed_last_token=bool(args.compat_refeed_last_token))
    inputs = build_inputs(model, tokenizer, args.prompt, args.image, share, pad_id)
    res, summary, first = benchmark_native(model, inputs, cfg, args.seed, tokenizer, args.benchmark_runs,
                                           row_offset=rank * share)
    if rank != 0:
        return {"native": {"summary": summary, "first_token_s": first, "tokens": res.tokens.cpu()}}
    print(format_summary_table("vlmrl sampler" + (f" ({world} processes)" if world > 1 else ""), summary, first))
    if res.texts:
        print("sample:", res.texts[0][:500])
    report: Dict[str, Any] = {"native": {"summary": summary, "first_token_s": first,
                                         "text": res.texts[0] if res.texts else "", "tokens": res.tokens.cpu()}}
    if args.compare_hf:
        try:
            hf = benchmark_hf(args.hf_model_name, args.prompt, args.image, args.max_new_tokens, args.temperature,
                              args.top_p, args.top_k, args.benchmark_runs, args.hf_dtype)
            print(format_summary_table("HuggingFace generate", hf["summary"], None))
            report["hf"] = hf
        except Exception as exc:  # the comparison is optional, as in the reference
            print(f"[eval] HF comparison skipped: {exc}")
            report["hf_error"] = str(exc)
    if args.plot_path:
        rows = {"vlmrl": summary}
        if "hf" in report:
            rows["hf"] = report["hf"]["summary"]
        report["plot"] = save_chart(args.plot_path, rows)
    if args.dump_metrics:
        os.makedirs(os.path.dirname(args.dump_metrics) or ".", exist_ok=True)
        with open(args.dump_metrics, "w", encoding="utf-8") as fh:
            json.dump({k: ({kk: vv for kk, vv in v.items() if kk != "tokens"} if isinstance(v, dict) else v)
                       for k, v in report.items()}, fh, indent=2, default=str)
    return report


if __name__ == "__main__":
    main()
