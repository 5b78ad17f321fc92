"""PPO / GRPO training CLI (reference ``core/train.py:1-457``).

``python -m vlmrl.core.train --model_dir=... --env_name=geospot --total_steps=1000``
(single GPU) or, one process per GPU,
``torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m vlmrl.core.train ...``.

Flags mirror the reference's ConfigDict (``core/train.py:44-100``) with the
same names and defaults, plus the flags of this framework's extensions:

* ``group_size`` / ``groups_per_batch`` — GRPO groups (``batch_size`` stays the
  number of prompts per iteration when ``groups_per_batch`` is not given);
* ``kl_ref_coef`` — k3 KL to a frozen copy of the initial policy;
* ``adv_norm`` — ``auto`` (batch normalisation as in the reference when
  ``group_size == 1``, per-group otherwise), ``batch``, ``group`` or ``none``;
* ``old_logprob_source`` — ``sampler`` (reference) or ``policy``;
* ``compat_refeed_last_token`` — rollouts start as the reference's sampler does (the last prompt
  token decoded a second time, prefill logits dropped); for parity runs;
* ``compat_decay_frozen`` — AdamW weight decay also shrinks the frozen vision tower every step, as the
  reference's optimizer does; for parity runs;
* ``preset`` — random-init architecture (``tiny``, ``qwen3vl_4b``, ...) when
  ``model_dir`` holds no weights;
* ``fsdp`` — shard optimizer state and gradients over the process group;
* ``fsdp_shard_params`` — also shard the decoder-layer bf16 weights (gathered inside the GEMMs);
* ``tp_rollout`` / ``tp_size`` — tensor-parallel rollout over groups of ``tp_size`` GPUs (0 = all).

Model loading accepts a converted checkpoint (``config.json`` + ``params.pkl``,
reference ``create_model_from_ckpt``) or a HuggingFace snapshot (safetensors).
Resume (``resume_path``) reads a ``train_state.pkl`` written by this CLI or the
reference (``{"train_state": {params, params_ema, opt_state, step}}``); saving
writes the same layout every ``save_interval`` iterations and at the end.
Metrics go to stdout, a JSONL file and, when installed and enabled, W&B.
"""

from __future__ import annotations

import json
import os
import sys
from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence

import torch

CONFIG: Dict[str, Any] = {
    # Logging / bookkeeping
    "wandb_project": "geospot",
    "wandb_name": "ppo-geospot-qwen3vl_4b",
    "wandb_group": "Default",
    "wandb_entity": "",
    "wandb_mode": "offline",
    "model_dir": "checkpoints/qwen3vl_4b",
    "save_dir": "runs/ppo-geospot-qwen3vl_4b",
    "save_interval": 20,
    "resume_path": "",
    "seed": 0,
    # Environment
    "env_name": "geospot",
    "env_split": "test",
    "env_max_samples": -1,
    "env_coord_tolerance_km": 25.0,
    "env_use_geo_shaping": 1,
    "env_geo_decay_km": 50.0,
    "env_country_weight": 0.2,
    "env_region_weight": 0.3,
    "env_city_weight": 0.5,
    # Training duration
    "total_steps": 1000,
    "batch_size": 16,
    "log_interval": 1,
    # Sampling / sequence knobs
    "temperature": 0.7,
    "top_p": 0.9,
    "top_k": 1024,
    "max_new_tokens": 64,
    "max_sequence_length": 2048,
    "vlm_min_pixels": -1,
    "vlm_max_pixels": -1,
    # PPO hyperparameters
    "clip_epsilon": 0.2,
    "entropy_coef": 0.0,
    "kl_coef": 0.0,
    "adaptive_kl": 1,
    "kl_target": 0.02,
    "kl_adapt_rate": 1.5,
    "kl_coef_min": 1e-5,
    "kl_coef_max": 0.5,
    "ppo_minibatch": 64,
    "ppo_epochs": 1,
    # Optimizer
    "optimizer": "adamw",
    "learning_rate": 1e-6,
    "weight_decay": 1e-2,
    "max_grad_norm": 1.0,
    "use_ema": 0,
    # Extensions of this framework
    "group_size": 1,
    "groups_per_batch": -1,
    "n_minibatches": 0,
    "kl_ref_coef": 0.0,
    "adv_norm": "auto",
    "old_logprob_source": "sampler",
    "compat_refeed_last_token": 0,
    "compat_decay_frozen": 0,
    "preset": "",
    "fsdp": 1,
    "fsdp_shard_params": 0,
    "tp_rollout": 0,
    "tp_size": 0,
    "metrics_path": "",
    "env_kwargs": "",
}

ALIASES = {"lr": "learning_rate", "steps": "total_steps"}


class RollingEnv:
    """Dataset-cursor wrapper over an environment (reference ``core/train.py:112-141``).

    ``reset(idx)`` resets task ``cursor + idx`` (modulo ``num_tasks``) and every
    ``step_list`` advances the cursor by the batch size and keeps the infos for
    the metric summary.  ``GRPOTrainer`` tracks its own cursor, so the CLI uses
    this wrapper only for its ``last_infos``.
    """

    def __init__(self, env):
        self._env = env
        self._cursor = 0
        self.last_infos: Dict[str, Any] = {}

    @property
    def num_tasks(self) -> int:
        return getattr(self._env, "num_tasks", -1)

    def reset(self, idx):
        total = self.num_tasks
        base = self._cursor + idx
        return self._env.reset(base % total if total and total > 0 else base)

    def step_list(self, states, actions):
        result = self._env.step_list(states, actions)
        self.last_infos = result[4]
        total = self.num_tasks
        self._cursor += len(states)
        if total and total > 0:
            self._cursor %= total
        return result

    def __getattr__(self, name):
        return getattr(self._env, name)


def resolve_pad_and_eos(tokenizer, spec) -> tuple:
    """(pad_id, eos_id) from the tokenizer, else from the model spec (reference ``core/train.py:144-153``)."""
    pad = getattr(tokenizer, "pad_token_id", None)
    if pad is None:
        pad = getattr(spec, "pad_token_id", 0)
    eos = getattr(tokenizer, "eos_token_id", None)
    if eos is None:
        eos = getattr(spec, "eos_token_id", None)
    return int(pad or 0), (int(eos) if eos is not None else None)


def resolve_image_pad_id(tokenizer, ckpt_dir: str, default: int = 151655) -> int:
    """Image placeholder id: tokenizer attribute, then ``config.json``, then 151655 (``core/train.py:156-175``)."""
    val = getattr(tokenizer, "image_token_id", None)
    if val is not None and int(val) >= 0:
        return int(val)
    special = getattr(tokenizer, "special_tokens_map", None)
    if isinstance(special, dict) and special.get("image_token_id") is not None:
        return int(special["image_token_id"])
    cfg_path = os.path.join(ckpt_dir or "", "config.json")
    if ckpt_dir and os.path.exists(cfg_path):
        with open(cfg_path, "r", encoding="utf-8") as fh:
            return int(json.load(fh).get("image_token_id", default))
    return int(default)


def _maybe(val) -> Optional[int]:
    return int(val) if int(val) > 0 else None


def load_policy(model_dir: str, preset: str, device, dtype=torch.bfloat16, seed: int = 0):
    """-> (Qwen3VLModel, fp32 master units or None).  Converted checkpoint, HF snapshot or random init."""
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.config import get_preset

    if model_dir and os.path.exists(os.path.join(model_dir, "params.pkl")):
        from vlmrl.models.qwen3vl.weights import create_model_from_ckpt

        cpu_model, _ = create_model_from_ckpt(model_dir)
        units = cpu_model.params.units
        return Qwen3VLModel(cpu_model.spec, units=units, device=device, dtype=dtype), units
    if model_dir and os.path.isdir(model_dir) and any(f.endswith(".safetensors") for f in os.listdir(model_dir)):
        from vlmrl.models.qwen3vl.weights import load_hf_units

        spec, units = load_hf_units(model_dir)
        return Qwen3VLModel(spec, units=units, device=device, dtype=dtype), units
    if not preset:
        raise FileNotFoundError(f"no params.pkl or safetensors under {model_dir!r}; pass --preset for a random init")
    return Qwen3VLModel(get_preset(preset), device=device, dtype=dtype, seed=seed), None


def build_env(args, tokenizer):
    """Environment from the flags (reference ``_build_env``, ``core/train.py:237-271``)."""
    from vlmrl.envs.base import create_env

    name = str(args.env_name or "").lower()
    kwargs: Dict[str, Any] = {}
    if name == "geospot":
        kwargs.update(split=str(args.env_split or "test"))
        if int(args.env_max_samples) > 0:
            kwargs["max_samples"] = int(args.env_max_samples)
    if args.env_kwargs:
        kwargs.update(json.loads(args.env_kwargs))
    return create_env(name, tokenizer, **kwargs)


def make_configs(args):
    """-> (TrainerConfig, AdamWConfig or AdafactorConfig) from parsed flags."""
    from vlmrl.core.optim import AdafactorConfig, AdamWConfig
    from vlmrl.core.ppo import TrainerConfig

    gs = max(1, int(args.group_size))
    groups = int(args.groups_per_batch) if int(args.groups_per_batch) > 0 else int(args.batch_size)
    adv = str(args.adv_norm)
    if adv == "auto":
        adv = "batch" if gs == 1 else "group"
    cfg = TrainerConfig(
        temperature=float(args.temperature),
        top_p=float(args.top_p) if 0.0 < float(args.top_p) < 1.0 else None,
        top_k=int(args.top_k) if int(args.top_k) > 0 else None,
        max_new_tokens=int(args.max_new_tokens),
        max_sequence_length=_maybe(args.max_sequence_length) or 0,
        clip_epsilon=float(args.clip_epsilon), entropy_coef=float(args.entropy_coef), kl_coef=float(args.kl_coef),
        adaptive_kl=bool(int(args.adaptive_kl)), kl_target=float(args.kl_target),
        kl_adapt_rate=float(args.kl_adapt_rate), kl_coef_min=float(args.kl_coef_min),
        kl_coef_max=float(args.kl_coef_max), ppo_minibatch=int(args.ppo_minibatch), ppo_epochs=int(args.ppo_epochs),
        n_minibatches=int(args.n_minibatches), groups_per_batch=groups, group_size=gs,
        kl_ref_coef=float(args.kl_ref_coef), adv_norm=adv, old_logprob_source=str(args.old_logprob_source),
        compat_refeed_last_token=bool(int(args.compat_refeed_last_token)),
        vlm_min_pixels=int(args.vlm_min_pixels), vlm_max_pixels=int(args.vlm_max_pixels))
    if str(args.optimizer).lower() == "adafactor":
        opt = AdafactorConfig(lr=float(args.learning_rate), weight_decay=float(args.weight_decay),
                              max_grad_norm=float(args.max_grad_norm))
    else:
        opt = AdamWConfig(lr=float(args.learning_rate), weight_decay=float(args.weight_decay),
                          max_grad_norm=float(args.max_grad_norm), decay_frozen=bool(int(args.compat_decay_frozen)))
    return cfg, opt


@dataclass
class RunState:
    trainer: Any
    iteration: int


def maybe_resume(trainer, resume_path: str, rank: int = 0) -> int:
    """Load ``resume_path`` into the trainer; returns the iteration to continue from (0 when nothing loaded)."""
    from vlmrl.utils.checkpoint import Checkpoint

    if not resume_path:
        return 0
    if not os.path.exists(resume_path):
        if rank == 0:
            print(f"[train] Resume path not found: {resume_path}")
        return 0
    try:
        data = Checkpoint(resume_path, parallel=False).load_as_dict()
        state = data.get("train_state", data)
        trainer.ts.load(state)
    except Exception as exc:  # unreadable or mismatched checkpoint: start fresh, as the reference does
        if rank == 0:
            print(f"[train] Failed to resume from {resume_path}: {exc}")
        return 0
    meta = data.get("metadata") or {}
    it = int(meta.get("step", trainer.ts.step - 1))
    trainer.iteration = it
    trainer.restore_state(meta.get("trainer"))
    if rank == 0:
        print(f"[train] Resumed state from {resume_path} at iteration {it}")
    return it


def maybe_save(trainer, save_dir: str, step: int, rank: int = 0) -> Optional[str]:
    """Write ``<save_dir>/train_state.pkl`` (collective under FSDP: every rank calls it, rank 0 writes)."""
    from vlmrl.utils.checkpoint import Checkpoint

    if not save_dir:
        return None
    state = trainer.ts.save()
    if rank != 0:
        return None
    os.makedirs(save_dir, exist_ok=True)
    path = os.path.join(save_dir, "train_state.pkl")
    cp = Checkpoint(path, parallel=False)
    cp.train_state = state
    cp.metadata = {"step": int(step), "trainer": trainer.state_dict()}
    cp.save()
    return path


def build_trainer(args, device=None, rank: int = 0, world: int = 1):
    """Model, tokenizer, environment, optimizer and trainer from parsed flags."""
    from vlmrl.core.trainer import GRPOTrainer
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.utils.tokenizer import load_tokenizer

    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    cfg, opt_cfg = make_configs(args)
    if world > 1 and int(args.fsdp):
        from vlmrl.models.qwen3vl.config import get_preset
        from vlmrl.parallel.fsdp import build_fsdp_models

        probe, units = load_policy(args.model_dir, args.preset, "cpu", torch.float32, seed=int(args.seed)) \
            if not args.preset else (None, None)
        spec = probe.spec if probe is not None else get_preset(args.preset)
        model, ref_model, ts = build_fsdp_models(spec, opt_cfg, seed=int(args.seed), device=device, units=units,
                                                 shard_params=bool(int(args.fsdp_shard_params)))
        master = None
    else:
        model, master = load_policy(args.model_dir, args.preset, device, dtype, seed=int(args.seed))
        text_units = {k: v for k, v in model.params.units.items() if k != "visual"}
        ref_model = Qwen3VLModel(model.spec, units=text_units, device=device, dtype=dtype) \
            if float(args.kl_ref_coef) > 0 else None
        ts = None
    tokenizer = load_tokenizer(args.model_dir if os.path.isdir(args.model_dir or "") else None,
                               vocab_size=model.spec.text.vocab_size)
    _, eos_id = resolve_pad_and_eos(tokenizer, model.spec)
    env = RollingEnv(build_env(args, tokenizer))
    trainer = GRPOTrainer(model, tokenizer, env, cfg, opt_cfg, ref_model=ref_model, seed=int(args.seed),
                          master=master, eos_id=eos_id, rank=rank, world_size=world, train_state=ts,
                          tp_rollout=bool(int(args.tp_rollout)) and world > 1, tp_size=int(args.tp_size))
    if int(args.use_ema) and trainer.ts.params_ema is None:
        trainer.ts.enable_ema()
    return trainer


def main(argv: Optional[Sequence[str]] = None) -> int:
    from vlmrl.parallel.dist import init_from_env
    from vlmrl.utils.configs import build_arg_parser
    from vlmrl.utils.wandb import MetricLogger, summarize_env_metrics

    args = build_arg_parser(CONFIG, ALIASES, description=__doc__).parse_args(argv)
    info = init_from_env()
    rank, world = info.rank, info.world_size
    device = torch.device("cuda", info.local_rank) if torch.cuda.is_available() else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    if rank == 0:
        print(f"[train] Loading model from {args.model_dir or args.preset}")
    trainer = build_trainer(args, device, rank, world)
    if world > 1:
        from vlmrl.parallel.watchdog import Heartbeat

        trainer.watchdog = Heartbeat()
    start = maybe_resume(trainer, str(args.resume_path or ""), rank)
    logger = None
    if rank == 0:
        path = args.metrics_path or (os.path.join(args.save_dir, "metrics.jsonl") if args.save_dir else "")
        logger = MetricLogger(path or None, config=vars(args), project=args.wandb_project, name=args.wandb_name,
                              group=args.wandb_group, entity=args.wandb_entity or None,
                              mode=str(args.wandb_mode).lower())
    total = int(args.total_steps)
    save_interval = int(args.save_interval)
    log_interval = max(1, int(args.log_interval))
    for step_idx in range(start, total):
        metrics = trainer.step()
        log_step = step_idx + 1
        metrics.update(summarize_env_metrics(getattr(trainer, "last_infos", {}) or {}))
        metrics["global_step"] = log_step
        if rank == 0 and log_step % log_interval == 0:
            preview = str(metrics.get("sample/text", "")).replace("\n", " ").strip()
            print("[train]", {"step": log_step, "reward": f"{metrics.get('reward/mean', 0.0):.3f}",
                              "approx_kl": f"{metrics.get('approx_kl', 0.0):.4f}",
                              "loss": f"{metrics.get('loss', 0.0):.4f}",
                              "entropy": f"{metrics.get('entropy', 0.0):.3f}", "response": preview})
            logger.log(metrics, step=log_step)
        if save_interval > 0 and log_step % save_interval == 0:
            maybe_save(trainer, args.save_dir, log_step, rank)
    maybe_save(trainer, args.save_dir, total, rank)
    if logger is not None:
        logger.close()
    if world > 1:
        import torch.distributed as dist

        trainer.watchdog.stop(leaving=True)
        dist.barrier()
        trainer.close()
        close = getattr(trainer.model.params, "close", None)
        if close is not None:
            close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
