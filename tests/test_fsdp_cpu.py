"""FSDP on 2 gloo CPU ranks: one GRPO step equals the single-process step on the same global batch."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _setup(groups):
    from vlmrl.core.optim import AdamWConfig
    from vlmrl.core.ppo import TrainerConfig
    from vlmrl.envs.base import create_env
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params
    from vlmrl.utils.tokenizer import ByteTokenizer

    spec = get_preset("tiny")
    units = init_params(spec, seed=0)
    tok = ByteTokenizer(spec.text.vocab_size)
    env = create_env("synthetic_parity", tok, image_size=64, prompt_tokens=16, num_tasks=64, seed=0, vocab_high=900)
    cfg = TrainerConfig(temperature=0.7, top_p=0.9, top_k=5, max_new_tokens=8, groups_per_batch=groups, group_size=4,
                        kl_ref_coef=0.05, n_minibatches=1, clip_epsilon=0.2, entropy_coef=0.01)
    return spec, units, tok, env, cfg, AdamWConfig(lr=1e-3, weight_decay=0.01, max_grad_norm=1.0)


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from vlmrl.core.trainer import GRPOTrainer
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.params import all_layouts, text_layouts
    from vlmrl.parallel.fsdp import FSDPOptimizer, FSDPParams
    from vlmrl.utils.train_state import TrainState

    spec, units, tok, env, cfg, adamw = _setup(groups=4)
    ref = Qwen3VLModel(spec, units={k: v for k, v in units.items() if k != "visual"}, dtype=torch.float32)
    fp = FSDPParams(all_layouts(spec), {k: v.clone() for k, v in units.items()}, dtype=torch.float32,
                    trainable=[l.name for l in text_layouts(spec)], replicate=["visual"])
    model = Qwen3VLModel(spec, params=fp, dtype=torch.float32)
    ts = TrainState(model, FSDPOptimizer(fp, adamw))
    trainer = GRPOTrainer(model, tok, env, cfg, adamw, ref_model=ref, seed=3, rank=rank, world_size=world,
                          train_state=ts)
    m = trainer.step()
    master = ts.optimizer.master_units()
    if rank == 0:
        torch.save({"master": {k: v.cpu() for k, v in master.items()}, "metrics": m}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_fsdp_two_ranks_matches_single_process(tmp_path):
    from vlmrl.core.trainer import GRPOTrainer
    from vlmrl.models.qwen3vl.api import Qwen3VLModel

    out = str(tmp_path / "fsdp.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    spec, units, tok, env, cfg, adamw = _setup(groups=4)
    model = Qwen3VLModel(spec, units=units, dtype=torch.float32)
    ref = Qwen3VLModel(spec, units={k: v for k, v in units.items() if k != "visual"}, dtype=torch.float32)
    single = GRPOTrainer(model, tok, env, cfg, adamw, ref_model=ref, seed=3)
    m = single.step()
    for k in ("loss", "loss_pg", "ref_kl", "entropy", "grad_norm", "reward/mean"):
        assert abs(m[k] - res["metrics"][k]) <= 1e-4 + 1e-4 * abs(m[k]), (k, m[k], res["metrics"][k])
    # AdamW's first update is ~lr*sign(g): gradients within rounding of zero may flip, so allow a fraction of lr
    for name, full in single.ts.optimizer.master.items():
        diff = (res["master"][name] - full.cpu()).abs()
        assert diff.max() <= 0.5 * adamw.lr, (name, float(diff.max()))
        assert (diff > 1e-6).float().mean() < 1e-3, name


def test_sharded_unit_small_leaf_ranges():
    """The leaves a sharded layer copies with one unit_gather: everything but the four GEMM matrices,
    16-byte aligned, neighbours merged across alignment padding, disjoint from the matrices."""
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import text_layouts
    from vlmrl.parallel.fsdp import GATHERED_LEAVES, _small_ranges

    lay = [l for l in text_layouts(get_preset("tiny")) if l.name == "layer0"][0]
    rng = _small_ranges(lay, GATHERED_LEAVES)
    assert all(a % 16 == 0 and b % 16 == 0 and a < b for a, b in rng)
    big = [(lay.offsets[k] * 2, (lay.offsets[k] + lay.spec(k).numel) * 2) for k in GATHERED_LEAVES]
    for a, b in rng:
        assert all(b <= s or a >= e for s, e in big)
    covered = set()
    for a, b in rng:
        covered.update(range(a, b, 2))
    for prm in lay.params:
        if prm.name not in GATHERED_LEAVES:
            lo = lay.offsets[prm.name] * 2
            assert set(range(lo, lo + prm.numel * 2, 2)) <= covered, prm.name
    # input_norm | qkv_b..k_norm | post_norm
    assert len(rng) == 3


def test_tp_partition_blocks_of_consecutive_ranks():
    from vlmrl.parallel.tp import tp_partition

    assert tp_partition(8, 2) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert tp_partition(4, 4) == [[0, 1, 2, 3]]
    with pytest.raises(ValueError):
        tp_partition(6, 4)
