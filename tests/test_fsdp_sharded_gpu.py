"""Sharded-parameter FSDP on 2 GPUs (NCCL ranks): decoder-layer weights are all-gathered inside the GEMMs
that consume them.  Log-probs, gradients, optimizer results and rollout-mode prefill must match the engine
that keeps the bf16 parameters gathered."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from tests.helpers import tiny_episodes
    from vlmrl import ops
    from vlmrl.core.optim import AdamWConfig
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import all_layouts, init_params, text_layouts
    from vlmrl.parallel.fsdp import FSDPOptimizer, FSDPParams

    dev = torch.device("cuda", rank)
    spec = get_preset("tiny")
    units = init_params(spec, seed=0, device=dev)
    cfg = AdamWConfig(lr=1e-3, weight_decay=0.01, max_grad_norm=1.0)
    res = {}
    engines = []
    for mode in ("gathered", "sharded"):
        fp = FSDPParams(all_layouts(spec), {k: v.clone() for k, v in units.items()}, dtype=torch.bfloat16,
                        trainable=[l.name for l in text_layouts(spec)], replicate=["visual"], comm="p2p",
                        shard_params=mode == "sharded")
        assert fp.comm == "p2p"
        assert bool(fp.sharded) == (mode == "sharded")
        engines.append(fp)
        opt = FSDPOptimizer(fp, cfg)
        m = Qwen3VLModel(spec, params=fp, dtype=torch.bfloat16, device=dev)
        out = {}
        for step in (1, 2):
            batch, _, _, _ = tiny_episodes(spec, m, n=4, seed=10 * step + rank, device=dev)
            lp, ent, ctx = m.token_logprobs(batch, save=True)
            out[f"lp{step}"] = lp.float().cpu()
            M = lp.numel()
            g1 = torch.randn(M, generator=torch.Generator().manual_seed(step)).to(dev)
            g2 = (torch.randn(M, generator=torch.Generator().manual_seed(step + 7)) * 0.1).to(dev)
            fp.zero_grads()
            with torch.no_grad():
                m.backward(ctx, g1, g2)
            fp.sync_grads()
            out[f"gshard{step}"] = {u: fp.grad_shards[u].cpu().clone() for u in fp.order}
            opt.step(step)
            ops.check_errors(rank)
            fp.verify_signals()
        out["master"] = {k: v.cpu() for k, v in opt.master_units().items()}
        out["full"] = {u: fp.get(u).float().cpu() for u in fp.order}
        # rollout mode: whole weights for prefill (sharded engine gathers them for the context)
        from vlmrl.core.batching import pack_prompts

        batch, _, seqs, plens = tiny_episodes(spec, m, n=3, prompt_text=9, action=4, seed=5, device=dev)
        prompts = [s[:p] for s, p in zip(seqs, plens)]
        pb, _ = pack_prompts(spec, prompts, [[(1, 4, 4)]] * 3, batch.vision, device=dev)
        with fp.inference_weights():
            cache = m.new_cache(3, 64)
            out["prefill"] = m.prefill(pb, cache, torch.arange(3, device=dev)).float().cpu()
        ops.check_errors(rank)
        res[mode] = out
        torch.cuda.synchronize()
    if rank == 0:
        torch.save(res, out_path)
    for fp in engines:
        fp.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_params_match_gathered(tmp_path):
    out = str(tmp_path / "sharded.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    a, b = res["gathered"], res["sharded"]
    for step in (1, 2):
        torch.testing.assert_close(b[f"lp{step}"], a[f"lp{step}"], atol=2e-3, rtol=1e-3)
        for u, g in a[f"gshard{step}"].items():
            torch.testing.assert_close(b[f"gshard{step}"][u], g, atol=1e-4, rtol=1e-3, msg=lambda s: f"grad {u}: {s}")
    for u, w in a["master"].items():
        torch.testing.assert_close(b["master"][u], w, atol=1e-5, rtol=1e-4, msg=lambda s: f"master {u}: {s}")
    for u, w in a["full"].items():
        # each engine's gathered bf16 parameters are exactly its fp32 master rounded: the in-GEMM / unit
        # gathers assembled every shard byte; across engines the two AdamW kernels may round one ulp apart
        for e in (a, b):
            torch.testing.assert_close(e["full"][u], e["master"][u].bfloat16().float(), atol=0, rtol=0,
                                       msg=lambda s: f"bf16 params {u} vs master: {s}")
        torch.testing.assert_close(b["full"][u], w, atol=1e-4, rtol=2 ** -7, msg=lambda s: f"bf16 params {u}: {s}")
    torch.testing.assert_close(b["prefill"], a["prefill"], atol=1e-3, rtol=1e-3)
