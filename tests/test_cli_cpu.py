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


def test_eval_cli_text_and_image(tmp_path):
    from PIL import Image

    from vlmrl.core import eval as eval_cli

    img = tmp_path / "img.png"
    Image.fromarray(np.random.default_rng(0).integers(0, 256, (64, 64, 3), dtype=np.uint8)).save(img)
    dump = tmp_path / "m.json"
    rep = eval_cli.main(["--preset=tiny", "--prompt=Where is this?", f"--image={img}", "--max_new_tokens=5",
                         "--benchmark_runs=2", "--batch=2", f"--dump_metrics={dump}",
                         f"--plot_path={tmp_path / 'chart.png'}"])
    s = rep["native"]["summary"]
    assert s["runs"] == 2 and s["tokens_total"] > 0 and "steady_throughput_mean" in s
    assert rep["native"]["first_token_s"] is not None
    assert json.load(open(dump))["native"]["summary"]["runs"] == 2
    rep = eval_cli.main(["--preset=tiny", "--prompt=hello", "--max_new_tokens=3", "--benchmark_runs=1"])
    assert rep["native"]["summary"]["runs"] == 1


def test_hf_to_jax_round_trip(tmp_path):
    from safetensors.torch import save_file

    from vlmrl.models.qwen3vl.config import spec_to_config
    from vlmrl.models.qwen3vl.weights import create_model_from_ckpt, units_to_hf_state_dict
    from vlmrl.utils import hf_to_jax

    spec, units, _ = tiny_model(seed=11)
    snap = tmp_path / "snap"
    snap.mkdir()
    json.dump(spec_to_config(spec), open(snap / "config.json", "w"))
    json.dump({"chat_template": "x"}, open(snap / "chat_template.json", "w"))
    sd = {k: v.contiguous() for k, v in units_to_hf_state_dict(spec, units).items()}
    save_file(sd, str(snap / "model.safetensors"))
    out = tmp_path / "ckpt"
    hf_to_jax.main([f"--model_dir={out}", f"--hf_dir={snap}"])
    assert (out / "params.pkl").exists() and (out / "config.json").exists() and (out / "chat_template.json").exists()
    model, params = create_model_from_ckpt(str(out))
    assert "params" not in params and len(params) > 0
    for name, t in units.items():
        torch.testing.assert_close(model.params.units[name], t, msg=lambda s: f"{name}: {s}")


def test_policy_token_logprobs_dense_matches_full_logits():
    from vlmrl.core.policy import build_rope, token_logprobs_vlm
    from vlmrl.models.qwen3vl.rope import mrope_cos_sin
    from helpers import tiny_episodes

    spec, units, m = tiny_model(seed=4)
    batch, counts, seqs, plens = tiny_episodes(spec, m, n=2, prompt_text=7, action=3)
    T = max(len(s) for s in seqs)
    tok = torch.zeros(2, T, dtype=torch.long)
    mask = torch.zeros(2, T - 1)
    for b, s in enumerate(seqs):
        tok[b, :len(s)] = torch.as_tensor(s)
        mask[b, :len(s) - 1] = 1
    grids = [[(1, 4, 4)], [(1, 4, 4)]]
    vis = batch.vision
    lp = token_logprobs_vlm(m, spec.image_token_id, tok, mask, vis, grids)
    n_img = 4
    for b, s in enumerate(seqs):
        rows = torch.arange(b * n_img, (b + 1) * n_img)
        logits = m.forward_vlm(torch.as_tensor(s[:-1])[None], vis.select(rows), [(1, 4, 4)])[0]
        exp = torch.log_softmax(logits.float(), -1).gather(-1, torch.as_tensor(s[1:])[:, None])[:, 0]
        torch.testing.assert_close(lp[b, :len(s) - 1], exp, atol=1e-4, rtol=1e-4)
        assert float(lp[b, len(s) - 1:].abs().sum()) == 0.0
    cos, sin = build_rope(spec, tok, grids)
    assert cos.shape == (2, T, spec.text.head_dim)
    assert torch.allclose(cos[0, 0], torch.ones(spec.text.head_dim))


def test_sharding_plans():
    from vlmrl.utils.sharding import create_sharding, get_local_slice, shard_axis

    shapes = {"embed": (151936, 2560), "norm": (2560,), "odd": (1001, 1003)}
    plan, rep, data, shard_data = create_sharding("fsdp", shapes, world=8)
    assert plan["embed"].axis == 0 and plan["norm"].axis is None and plan["odd"].axis is None
    assert shard_axis((7, 4096, 1024), 2, 8) == 1
    x = torch.arange(16).reshape(8, 2)
    assert torch.equal(shard_data(x), x[0:1])  # rank 0 of the 8 the plan was made for
    assert torch.equal(shard_data(x[:3]), x[:3])  # not divisible: kept whole
    assert torch.equal(get_local_slice(x, world=4, rank=1), x[2:4])
    plan, *_ = create_sharding("dp")
    assert plan.axis is None


def test_rollout_cli(capsys):
    from vlmrl.core import rollout

    rewards = rollout.main(["--preset=tiny", "--env_name=synthetic_parity", "--episodes=5", "--batch_size=2",
                            "--max_new_tokens=4", "--top_k=8"])
    assert len(rewards) == 5
    out = capsys.readouterr().out
    assert "[episode 4]" in out and "Collected 5 episodes" in out


def _eval_rank(rank, world, port, out_dir):
    import os

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    from vlmrl.core import eval as eval_cli

    rep = eval_cli.main(["--preset=tiny", "--prompt=hello there", "--max_new_tokens=6", "--benchmark_runs=1",
                         "--batch=4", "--temperature=0.9"])
    torch.save({"tokens": rep["native"]["tokens"], "summary": rep["native"]["summary"]}, f"{out_dir}/r{rank}.pt")
    dist.destroy_process_group()


def test_eval_cli_data_parallel_matches_one_process(tmp_path):
    """Two gloo ranks split --batch 4: each samples its rows with their global row ids, so together they draw
    the single-process tokens; throughput counts every rank's tokens."""
    import socket

    import torch.multiprocessing as mp

    from vlmrl.core import eval as eval_cli

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_eval_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    single = eval_cli.main(["--preset=tiny", "--prompt=hello there", "--max_new_tokens=6", "--benchmark_runs=1",
                            "--batch=4", "--temperature=0.9"])
    parts = [torch.load(tmp_path / f"r{r}.pt") for r in range(2)]
    assert torch.equal(torch.cat([p["tokens"] for p in parts]), single["native"]["tokens"])
    assert parts[0]["summary"]["tokens_total"] == single["native"]["summary"]["tokens_total"]
