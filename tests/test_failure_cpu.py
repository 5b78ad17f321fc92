"""Failure detection on the host (gloo CPU ranks): heartbeats, a rank that dies or leaves, a collective with a
missing peer, an environment that raises, an unreadable checkpoint.  No GPU is involved."""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=20):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _hb_worker(rank, world, port, mode, out):
    dist = _init(rank, world, port)
    from vlmrl.parallel.watchdog import Heartbeat, RankFailure

    hb = Heartbeat(interval=0.05, timeout=0.6, grace=5.0)
    dist.barrier()
    if rank == 0:
        hb.check()                     # everyone alive at first
    dist.barrier()
    if rank == 1:
        if mode == "dies":
            hb.stop()                  # silent: the process stays alive but stops beating
            time.sleep(3.0)
        else:
            hb.stop(leaving=True)
            time.sleep(1.0)
        return
    t0 = time.time()
    err = None
    while time.time() - t0 < 5.0:
        try:
            hb.check()
        except RankFailure as exc:
            err = exc
            break
        time.sleep(0.05)
    torch.save({"ranks": err.ranks if err else None, "msg": str(err), "after": time.time() - t0}, out)
    hb.stop()


@pytest.mark.parametrize("mode", ["dies", "leaves"])
def test_heartbeat_reports_silent_or_departed_rank(tmp_path, mode):
    out = str(tmp_path / "hb.pt")
    mp.start_processes(_hb_worker, args=(2, _free_port(), mode, out), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    assert res["ranks"] == [1], res
    assert ("left" in res["msg"]) == (mode == "leaves")
    assert res["after"] < 4.0


def _dead_peer_worker(rank, world, port, out):
    dist = _init(rank, world, port, timeout_s=3)
    t = torch.ones(4)
    dist.all_reduce(t)                 # one healthy collective
    if rank == 1:
        os._exit(0)                    # dies between steps, before the next collective
    t0 = time.time()
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as exc:           # gloo: connection closed / timeout
        outcome = type(exc).__name__
    torch.save({"outcome": outcome, "after": time.time() - t0}, out)
    os._exit(0)


def test_collective_with_dead_peer_fails_fast(tmp_path):
    out = str(tmp_path / "dead.pt")
    ctx = mp.start_processes(_dead_peer_worker, args=(2, _free_port(), out), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 60
    while not ctx.join(timeout=1) and time.time() < deadline:
        pass
    res = torch.load(out)
    assert res["outcome"] != "completed"
    assert res["after"] < 30


class _Boom(RuntimeError):
    pass


def test_env_error_propagates_from_trainer_step():
    from vlmrl.core.optim import AdamWConfig
    from vlmrl.core.ppo import TrainerConfig
    from vlmrl.core.trainer import GRPOTrainer
    from vlmrl.envs.base import create_env
    from vlmrl.utils.tokenizer import ByteTokenizer

    from helpers import tiny_model

    spec, units, m = tiny_model(seed=2)
    env = create_env("synthetic_parity", ByteTokenizer(spec.text.vocab_size), num_tasks=8)

    def broken(states, actions):
        raise _Boom("reward service unavailable")

    env.step_list = broken
    tr = GRPOTrainer(m, ByteTokenizer(spec.text.vocab_size), env,
                     TrainerConfig(max_new_tokens=3, groups_per_batch=2, group_size=2, top_k=8), AdamWConfig())
    with pytest.raises(_Boom):
        tr.step()


def test_unreadable_checkpoint_resume_starts_fresh(tmp_path, capsys):
    from vlmrl.core import train as train_cli

    bad = tmp_path / "train_state.pkl"
    bad.write_bytes(b"\x80\x04 not a pickle")
    args = ["--model_dir=", "--preset=tiny", "--env_name=synthetic_parity", "--batch_size=2", "--group_size=2",
            "--max_new_tokens=3", "--top_k=8", "--wandb_mode=disabled", "--total_steps=1", f"--resume_path={bad}",
            f"--save_dir={tmp_path / 'run'}"]
    assert train_cli.main(args) == 0
    assert "Failed to resume" in capsys.readouterr().out


def test_resume_restores_rng_and_cursor(tmp_path):
    import pickle

    from vlmrl.core import train as train_cli

    base = ["--model_dir=", "--preset=tiny", "--env_name=synthetic_parity", "--batch_size=2", "--group_size=2",
            "--max_new_tokens=3", "--top_k=8", "--wandb_mode=disabled"]
    train_cli.main(base + ["--total_steps=2", f"--save_dir={tmp_path / 'a'}", "--save_interval=1"])
    meta = pickle.load(open(tmp_path / "a" / "train_state.pkl", "rb"))["metadata"]
    assert meta["trainer"]["cursor"] == 4 and meta["trainer"]["iteration"] == 2
