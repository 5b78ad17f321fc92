"""CPU tests for the training CLI (flags, save, resume) and the Adafactor optimizer."""

import json
import os
import pickle

import numpy as np
import torch

from vlmrl.core import train as train_cli
from vlmrl.core.optim import AdafactorConfig, LocalAdafactor, leaf_views
from vlmrl.models.qwen3vl.model import LocalParams

from helpers import tiny_model

ARGS = ["--model_dir=", "--preset=tiny", "--env_name=synthetic_parity", "--batch_size=2", "--group_size=2",
        "--max_new_tokens=4", "--top_k=8", "--learning_rate=1e-4", "--wandb_mode=disabled"]


def test_train_cli_save_and_resume(tmp_path):
    save = str(tmp_path / "run")
    assert train_cli.main(ARGS + [f"--save_dir={save}", "--total_steps=2", "--save_interval=1"]) == 0
    ckpt = os.path.join(save, "train_state.pkl")
    with open(ckpt, "rb") as fh:
        data = pickle.load(fh)
    st = data["train_state"]
    assert set(st) == {"params", "params_ema", "opt_state", "step"}
    assert st["step"] == 3 and data["metadata"]["step"] == 2
    rows = [json.loads(l) for l in open(os.path.join(save, "metrics.jsonl"))]
    assert [r["step"] for r in rows] == [1, 2] and all("loss" in r for r in rows)
    # resume: continues at iteration 2 and stops after one more step
    save2 = str(tmp_path / "run2")
    assert train_cli.main(ARGS + [f"--save_dir={save2}", "--total_steps=3", f"--resume_path={ckpt}"]) == 0
    with open(os.path.join(save2, "train_state.pkl"), "rb") as fh:
        st2 = pickle.load(fh)["train_state"]
    assert st2["step"] == 4
    rows2 = [json.loads(l) for l in open(os.path.join(save2, "metrics.jsonl"))]
    assert [r["step"] for r in rows2] == [3]


def test_flags_match_reference_names():
    ref_keys = {"wandb_project", "wandb_name", "wandb_group", "wandb_entity", "wandb_mode", "model_dir", "save_dir",
                "save_interval", "resume_path", "seed", "env_name", "env_split", "env_max_samples",
                "env_coord_tolerance_km", "env_use_geo_shaping", "env_geo_decay_km", "env_country_weight",
                "env_region_weight", "env_city_weight", "total_steps", "batch_size", "log_interval", "temperature",
                "top_p", "top_k", "max_new_tokens", "max_sequence_length", "vlm_min_pixels", "vlm_max_pixels",
                "clip_epsilon", "entropy_coef", "kl_coef", "adaptive_kl", "kl_target", "kl_adapt_rate",
                "kl_coef_min", "kl_coef_max", "ppo_minibatch", "ppo_epochs", "optimizer", "learning_rate",
                "weight_decay", "max_grad_norm", "use_ema"}
    assert ref_keys <= set(train_cli.CONFIG)
    args = train_cli.build_arg_parser_for_tests(["--lr=3e-5", "--top_p=1.0", "--top_k=0"]) \
        if hasattr(train_cli, "build_arg_parser_for_tests") else None
    from vlmrl.utils.configs import build_arg_parser

    args = build_arg_parser(train_cli.CONFIG, train_cli.ALIASES).parse_args(["--lr=3e-5", "--top_p=1.0", "--top_k=0"])
    cfg, opt = train_cli.make_configs(args)
    assert opt.lr == 3e-5 and cfg.top_p is None and cfg.top_k is None and cfg.adv_norm == "batch"


def _adafactor_leaf_np(p, g, lr, wd, steps):
    """Independent NumPy statement of the Adafactor leaf update for `steps` identical gradients."""
    p = p.astype(np.float64).copy()
    if p.ndim == 2 and min(p.shape) >= 32:
        big = int(np.argmax(p.shape))
        small = 1 - big
        vr = np.zeros(p.shape[small])
        vc = np.zeros(p.shape[big])
    else:
        v = np.zeros_like(p)
    for t in range(steps):
        beta = 1.0 - (t + 1.0) ** -0.8
        g2 = g.astype(np.float64) ** 2 + 1e-30
        if p.ndim == 2 and min(p.shape) >= 32:
            vr = beta * vr + (1 - beta) * g2.mean(axis=big)
            vc = beta * vc + (1 - beta) * g2.mean(axis=small)
            denom = np.expand_dims(vr, big) * np.expand_dims(vc, small) / vr.mean()
            u = g / np.sqrt(denom)
        else:
            v = beta * v + (1 - beta) * g2
            u = g / np.sqrt(v)
        u = u / max(1.0, np.sqrt((u ** 2).mean()))
        u = u * lr * max(np.sqrt((p ** 2).mean()), 1e-3)
        p = p - (u + wd * p)
    return p


def test_adafactor_matches_numpy_statement():
    spec, units, model = tiny_model(seed=3)
    params = LocalParams({k: v.clone() for k, v in units.items()}, trainable=["layer0"])
    cfg = AdafactorConfig(lr=1e-2, weight_decay=1e-2, max_grad_norm=0.0)
    opt = LocalAdafactor(params, cfg, spec=spec)
    g = torch.randn(params.units["layer0"].numel(), generator=torch.Generator().manual_seed(0))
    before = {n: v.clone().numpy() for n, v in leaf_views(spec, "layer0", opt.master["layer0"])}
    gl = {n: v.clone().numpy() for n, v in leaf_views(spec, "layer0", g)}
    for step in (1, 2):
        params.grads["layer0"].copy_(g)
        opt.step(step)
    after = dict(leaf_views(spec, "layer0", opt.master["layer0"]))
    for name, p0 in before.items():
        exp = _adafactor_leaf_np(p0, gl[name], 1e-2, 1e-2, 2)
        np.testing.assert_allclose(after[name].numpy(), exp, rtol=2e-4, atol=1e-6, err_msg=name)
