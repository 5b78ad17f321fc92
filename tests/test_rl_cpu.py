"""CPU end-to-end: envs, rollout, GRPO update on the tiny model (fp32)."""

import numpy as np
import pytest
import torch

from vlmrl.core.grpo import group_advantages, ppo_loss
from vlmrl.core.kl import AdaptiveKL
from vlmrl.core.optim import AdamWConfig
from vlmrl.core.ppo import TrainerConfig
from vlmrl.core.trainer import GRPOTrainer
from vlmrl.envs.base import create_env
from vlmrl.models.qwen3vl.api import Qwen3VLModel
from vlmrl.models.qwen3vl.config import get_preset
from vlmrl.models.qwen3vl.params import init_params, text_layouts
from vlmrl.utils.tokenizer import ByteTokenizer


def _tiny_trainer(**over):
    spec = get_preset("tiny")
    units = init_params(spec, seed=0)
    model = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    ref = Qwen3VLModel(spec, units={k: v for k, v in units.items() if k != "visual"}, dtype=torch.float32)
    tok = ByteTokenizer(spec.text.vocab_size)
    env = create_env("synthetic_parity", tok, image_size=64, prompt_tokens=16, num_tasks=64, seed=0,
                     vocab_high=900)
    cfg = TrainerConfig(temperature=0.7, top_p=0.9, top_k=5, max_new_tokens=16, groups_per_batch=4, group_size=4,
                        kl_ref_coef=0.01, n_minibatches=2, clip_epsilon=0.2)
    for k, v in over.items():
        setattr(cfg, k, v)
    return GRPOTrainer(model, tok, env, cfg, AdamWConfig(lr=5e-7), ref_model=ref, seed=0), units


def test_group_advantages():
    r = torch.tensor([1.0, 0.0, 1.0, 0.0, 2.0, 2.0])
    a = group_advantages(r, 2)
    assert torch.allclose(a.view(3, 2).mean(1), torch.zeros(3), atol=1e-6)
    assert a[4] == 0 and a[5] == 0
    b = group_advantages(r, 1, mode="batch")
    assert abs(float(b.mean())) < 1e-6


def test_ppo_loss_ratio_one_gradient():
    lp = torch.tensor([-1.0, -2.0, -0.5])
    adv = torch.tensor([1.0, -1.0, 0.5])
    loss, g_lp, g_ent, m = ppo_loss(lp, torch.zeros(3), lp.clone(), adv, clip_epsilon=0.2)
    # at ratio 1 the policy-gradient term is -A * r, whose gradient wrt logp is -A / denom
    torch.testing.assert_close(g_lp, -adv / 3)
    assert float(m["clip_fraction"]) == 0.0 and abs(float(m["approx_kl"])) < 1e-7


def test_adaptive_kl():
    c = AdaptiveKL(target=0.02, rate=1.5)
    assert c.update(0.1, 0.01) == pytest.approx(0.015)
    assert c.update(0.001, 0.01) == pytest.approx(0.01 / 1.5)
    assert c.update(1.0, 0.01) == pytest.approx(min(0.5, 0.01 * 1.5 ** 3))


def test_grpo_step_tiny_cpu():
    trainer, units = _tiny_trainer()
    m = trainer.step()
    assert trainer.ts.step == 3  # two minibatches -> two optimizer steps
    for k in ("loss", "loss_pg", "ref_kl", "approx_kl", "grad_norm", "reward/mean", "entropy"):
        assert k in m and np.isfinite(m[k]), k
    # parameters moved, the frozen reference did not
    moved = any(not torch.equal(trainer.model.params.units[l.name], units[l.name])
                for l in text_layouts(trainer.model.spec))
    assert moved
    assert all(torch.equal(trainer.ref_model.params.units[k], units[k]) for k in trainer.ref_model.params.units)
    # first minibatch starts exactly on-policy
    assert abs(m["approx_kl"]) < 1e-3


def test_train_state_roundtrip(tmp_path):
    from vlmrl.utils.checkpoint import Checkpoint

    trainer, _ = _tiny_trainer(n_minibatches=1)
    trainer.step()
    ck = Checkpoint(str(tmp_path / "train_state.pkl"), parallel=False)
    ck.train_state = trainer.ts
    ck.metadata = {"step": trainer.ts.step}
    ck.save()
    data = Checkpoint(str(tmp_path / "train_state.pkl"), parallel=False).load_as_dict()
    assert set(data["train_state"]) == {"params", "params_ema", "opt_state", "step"}
    assert "layers_0" in data["train_state"]["params"] and "lm_head" in data["train_state"]["params"]
    adam = data["train_state"]["opt_state"][1][0]
    assert adam.mu["layers_0"]["attn"]["q_proj"]["kernel"].shape == data["train_state"]["params"]["layers_0"]["attn"]["q_proj"]["kernel"].shape
    t2, _ = _tiny_trainer(n_minibatches=1)
    t2.ts.load(data["train_state"])
    for name, buf in trainer.ts.optimizer.master.items():
        torch.testing.assert_close(t2.ts.optimizer.master[name], buf)
    assert t2.ts.step == trainer.ts.step


def test_rollout_only_tiny_cpu():
    """GRPOTrainer.rollout: the inference workload — rollout and rewards, no optimizer step."""
    trainer, units = _tiny_trainer()
    m = trainer.rollout()
    assert trainer.ts.step == 1  # no update ran
    assert m["sequences"] == 16 and 0 < m["tokens/generated"] <= 16 * 16
    assert np.isfinite(m["reward/mean"]) and "time/rollout_ms" in m
    assert all(torch.equal(trainer.model.params.units[l.name], units[l.name]) for l in text_layouts(trainer.model.spec))
    # the dataset cursor advances as for a training step
    assert trainer.cursor == 4


def test_grpo_update_with_nonzero_geodesic_rewards():
    """reward -> advantage -> loss -> gradient with the geodesic reward actually varying.

    Random-init weights never emit parseable coordinates, so a plain rollout scores 0 everywhere.  Here the
    sampled responses are replaced by byte-encoded answers at known distances from each group's target (exact,
    ~150 km, ~2000 km, unparseable), and the whole trainer step runs on them: rewards must fall with
    distance, advantages must be non-zero and centred per group, and the update must move the weights."""
    from vlmrl.core.sampling import Generator

    spec = get_preset("tiny")
    units = init_params(spec, seed=0)
    model = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    ref = Qwen3VLModel(spec, units={k: v for k, v in units.items() if k != "visual"}, dtype=torch.float32)
    tok = ByteTokenizer(spec.text.vocab_size)
    env = create_env("synthetic_geo", tok, image_size=64, prompt_tokens=16, num_tasks=64, seed=0, vocab_high=900)
    G, gs, max_new = 2, 4, 48
    cfg = TrainerConfig(temperature=0.7, top_p=0.9, top_k=5, max_new_tokens=max_new, groups_per_batch=G,
                        group_size=gs, kl_ref_coef=0.01, n_minibatches=1, clip_epsilon=0.2)
    trainer = GRPOTrainer(model, tok, env, cfg, AdamWConfig(lr=1e-4), ref_model=ref, seed=0)
    targets = [env.reset(trainer.cursor + g)[0].target for g in range(G)]
    offsets = [(0.0, 0.0), (1.0, 1.0), (15.0, 12.0), None]   # degrees; None: prose without coordinates

    real = Generator.generate

    def crafted(self, *a, **kw):
        res = real(self, *a, **kw)
        toks = torch.full_like(res.tokens, tok.pad_token_id)
        lens = torch.zeros_like(res.lengths)
        for g in range(G):
            c = targets[g]
            for j, off in enumerate(offsets):
                text = ("I cannot tell." if off is None else
                        f"Latitude: {max(-90.0, min(90.0, c.lat + off[0])):.4f}\nLongitude: {c.lon + off[1]:.4f}")
                ids = tok.encode(text)[:max_new]
                b = g * gs + j
                toks[b, :len(ids)] = torch.tensor(ids, dtype=toks.dtype)
                lens[b] = len(ids)
        res.tokens, res.lengths = toks, lens
        return res

    Generator.generate = crafted
    try:
        m = trainer.step()
    finally:
        Generator.generate = real
    cr = trainer.last_collect
    r = cr.rewards.view(G, gs)
    assert torch.all(r[:, 0] > r[:, 1]) and torch.all(r[:, 1] > r[:, 2]) and torch.all(r[:, 3] == 0), r
    assert torch.allclose(r[:, 0], torch.ones(G), atol=1e-3)   # 4-decimal coordinates: metres off
    adv = cr.advantages.view(G, gs).cpu()
    assert torch.allclose(adv.mean(1), torch.zeros(G), atol=1e-5)
    assert torch.all(adv[:, 0] > 0) and torch.all(adv[:, 3] < 0)
    assert m["reward/mean"] > 0.2
    for k in ("loss", "loss_pg", "grad_norm"):
        assert np.isfinite(m[k]), k
    assert m["grad_norm"] > 0 and abs(m["loss_pg"]) > 0
    moved = any(not torch.equal(trainer.model.params.units[l.name], units[l.name])
                for l in text_layouts(trainer.model.spec))
    assert moved
