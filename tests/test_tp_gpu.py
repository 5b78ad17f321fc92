"""Tensor-parallel decode on 2 GPUs: the NVLink all-reduce inside the consumer kernels reproduces the
single-GPU decode logits, both ranks sample identical tokens, and the vocab-parallel lm_head + sampler
draws on every rank the token and log-probability the single-GPU fused sampler draws."""

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


def _worker(rank, world, port, out_path, preset):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import datetime

    import numpy as np
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from vlmrl import ops
    from vlmrl.core.batching import pack_prompts
    from vlmrl.core.sampling import Generator
    from vlmrl.core.types import SamplingConfig
    from vlmrl.models.qwen3vl.api import Qwen3VLModel
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import init_params
    from vlmrl.parallel.tp import TPDecoder

    dev = torch.device("cuda", rank)
    spec = get_preset(preset)
    units = init_params(spec, seed=3, device=dev)
    m = Qwen3VLModel(spec, units=units, dtype=torch.bfloat16, device=dev)
    tp = TPDecoder(m, max_batch=8)
    tp.refresh()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 900, n) for n in (17, 30, 5, 44)]
    pb, deltas = pack_prompts(spec, prompts, [[]] * 4, None, device=dev)
    full = m.new_cache(4, 128)
    m.prefill(pb, full, torch.arange(4, device=dev))
    local = tp.new_cache(4, 128)
    tp.load_cache(full, local, 64)
    dl = torch.from_numpy(deltas).to(dev)
    tok = torch.tensor([5, 6, 7, 8], device=dev)
    ref_logits, tp_logits = [], []
    for step in range(3):
        ref_logits.append(m.decode_step(tok, full, dl).float().cpu())
        tp_logits.append(tp.decode_step(tok, local, dl).float().cpu())
        tok = (tok * 7 + step) % 900
    ops.check_errors(rank)
    # full sampler through the generator with CUDA graphs: every rank must agree token for token
    gen = Generator(m, tp=tp)
    cfg = SamplingConfig(temperature=0.8, top_k=20, top_p=0.95, eos_id=None, pad_id=0, max_new_tokens=12)
    res = gen.generate(prompts, [[]] * 4, None, cfg, seed=11, group_size=2)
    ops.check_errors(rank)
    toks = res.tokens.cpu()
    gathered = [torch.zeros_like(toks) for _ in range(world)]
    dist.all_gather_object(gathered, toks)
    # vocab-parallel lm_head + sampler on the same rows: every rank draws what the single-GPU fused sampler
    # draws from the whole vocabulary (the shard GEMMs give the same logits per column)
    from vlmrl.ops._ext import ext

    g = torch.Generator(device=dev).manual_seed(4)
    hn = torch.randn(8, spec.text.hidden_size, generator=g, device=dev).to(torch.bfloat16)
    lm = m.decoder._w(m.params, "head")["lm_head"]
    seed_t = torch.tensor([123], dtype=torch.int64, device=dev)
    fused = []
    for step in range(3):
        step_t = torch.tensor([step], dtype=torch.int64, device=dev)
        ref_tok, ref_lp = ops.lm_head_sample(hn, lm, temperature=0.8, top_k=5, top_p=0.9, seed=seed_t, step=step_t)
        ext().tp_step_begin(tp.epoch.data_ptr(), rank)   # a new exchange tag, as every decode step does
        tp_tok = torch.empty(8, dtype=torch.int64, device=dev)
        tp_lp = torch.empty(8, dtype=torch.float32, device=dev)
        ext().lm_head_sample_tp(hn, tp.lm_w, tp.v0, tp_tok, tp_lp, step_t, seed_t, 0.8, 5, 0.9, 0,
                                tp.samp_slots.ptrs, 0, tp.epoch.data_ptr(), rank)
        fused.append((ref_tok.cpu(), ref_lp.cpu(), tp_tok.cpu(), tp_lp.cpu()))
    ops.check_errors(rank)
    fused_all = [None] * world
    dist.all_gather_object(fused_all, fused)
    if rank == 0:
        torch.save({"ref": ref_logits, "tp": tp_logits, "tokens": gathered, "fused": fused_all}, out_path)
    dist.barrier()
    tp.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("preset", ["tiny", "tiny_qwen25"])
def test_tp_decode_matches_single_gpu(tmp_path, preset):
    out = str(tmp_path / "tp.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out, preset), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    for a, b in zip(res["tp"], res["ref"]):
        assert (a - b).abs().max().item() < 0.05 * max(1.0, b.abs().max().item())
    assert torch.equal(res["tokens"][0], res["tokens"][1])
    for per_rank in res["fused"]:
        for ref_tok, ref_lp, tp_tok, tp_lp in per_rank:
            assert torch.equal(ref_tok, tp_tok)
            torch.testing.assert_close(ref_lp, tp_lp, atol=1e-5, rtol=1e-5)
