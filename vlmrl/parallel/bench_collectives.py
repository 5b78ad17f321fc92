"""Device-timed microbenchmarks of the peer-memory collective kernels (one process per GPU).

``torchrun --nproc-per-node N -m vlmrl.parallel.bench_collectives`` times, with
CUDA events on the launching stream and the max over ranks:

* ``rs_pull``      — gradient reduce-scatter of one decoder layer unit (fp32), the kernel of the FSDP
                     ``p2p`` path, against ``reduce_scatter_tensor`` (NCCL) on the same buffer;
* ``adamw_push``   — sharded AdamW + bf16 all-gather by peer stores for one layer, against NCCL
                     ``all_gather_into_tensor`` of the same bf16 shard (plus the local AdamW kernel);
* ``dec_residual_norm_tp`` — the tensor-parallel decode consumer (batch 64 x 2560 partials all-reduced
                     in the kernel), against an NCCL all-reduce of the same fp32 rows;
* ``gemm_gather``  — the FSDP (sharded-parameter) forward GEMM of the gate/up projection, 5112 tokens x
                     2560 -> 19456, whose weight is all-gathered from the ranks' shards inside the GEMM,
                     against NCCL ``all_gather_into_tensor`` followed by the same GEMM; also the dgrad form
                     (MN-major weight operand).

Roofline: bytes that must cross NVLink per rank / 770 GB/s (the measured peer-copy bandwidth per
direction), or for the GEMM cases the slower of that and FLOPs at the measured bf16 burst peak (HBM-side
terms at the measured copy bandwidth; both from MEASURED_PEAKS.json, else the fallback figures); the
achieved fraction is that time divided by the measured time.  Prints one JSON line per case on rank 0.
"""

from __future__ import annotations

import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _peaks():
    from vlmrl.ops.bench_kernels import peaks

    return peaks()


GEMM_TFLOPS, HBM_GBS, PEAK_SOURCE = _peaks()


def _timed(fn, iters: int = 20, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from vlmrl import ops
    from vlmrl.ops._ext import ext
    from vlmrl.parallel.symm import SymmetricBuffer

    W, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", local)
    out = []

    # ---- reduce-scatter of one layer's fp32 gradient (4B model: 101M parameters -> padded)
    n_full = (101 * 2 ** 20 // (128 * W)) * 128 * W
    n = n_full // W
    grads = SymmetricBuffer(n_full * 4, None, dev)
    sig = SymmetricBuffer(4 * W * 8, None, dev)
    g = grads.view(0, (n_full,), torch.float32)
    g.normal_()
    shard = torch.zeros(n, device=dev)
    epoch = [0]

    link_bytes = (W - 1) * n * 4           # this rank pulls its shard from every peer
    ideal = link_bytes / (LINK_GBS * 1e9) * 1e3
    for ctas in (0, 296, 592):
        def rs_p2p(ctas=ctas):
            epoch[0] += 1
            ext().rs_pull(grads.ptrs, 0, r * n, shard, False, sig.ptrs, 0, epoch[0], r, ctas)

        ms = _timed(rs_p2p)
        ops.check_errors(local)
        out.append({"case": f"rs_pull_fp32_{n_full}", "ctas": ctas or "sms", "world": W, "ms": round(ms, 4),
                    "link_GBps": round(link_bytes / ms / 1e6, 1), "roofline_ms": round(ideal, 4),
                    "frac_of_roofline": round(ideal / ms, 3)})
    full = torch.randn(n_full, device=dev)
    ms_nccl = _timed(lambda: dist.reduce_scatter_tensor(shard, full))
    out.append({"case": f"nccl_reduce_scatter_fp32_{n_full}", "world": W, "ms": round(ms_nccl, 4),
                "frac_of_roofline": round(ideal / ms_nccl, 3)})

    # ---- AdamW on the shard + bf16 push into every rank's gathered buffer
    params = SymmetricBuffer(n_full * 2, None, dev)
    p32, m, v = torch.randn(n, device=dev), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    gs = torch.randn(n, device=dev)
    scale = torch.ones(1, device=dev)
    target = [0]

    def push():
        grid = ext().adamw_push(p32, gs, m, v, params.ptrs, r * n * 2, scale, 1e-7, 0.9, 0.999, 1e-8, 0.01, 1,
                                sig.ptrs, 1, r)
        target[0] += int(grid)
        ext().peer_wait(sig.local, 1, target[0], r, W, local)

    ms = _timed(push)
    ops.check_errors(local)
    link_bytes = (W - 1) * n * 2             # this rank's bf16 shard stored into every peer
    local_bytes = n * (4 * 4 + 3 * 4 + 2)    # AdamW reads p, g, m, v and writes p, m, v, own bf16
    ideal = max(link_bytes / (LINK_GBS * 1e9), local_bytes / (HBM_GBS * 1e9)) * 1e3
    out.append({"case": f"adamw_push_{n_full}", "world": W, "ms": round(ms, 4), "roofline_ms": round(ideal, 4),
                "frac_of_roofline": round(ideal / ms, 3)})
    gathered = torch.empty(n_full, dtype=torch.bfloat16, device=dev)
    ph = torch.empty(n, dtype=torch.bfloat16, device=dev)

    def nccl_path():
        ops.adamw_(p32, gs, m, v, lr=1e-7, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=1,
                   grad_scale=scale, p_half=ph)
        dist.all_gather_into_tensor(gathered, ph)

    ms_nccl = _timed(nccl_path)
    out.append({"case": f"adamw_then_nccl_all_gather_{n_full}", "world": W, "ms": round(ms_nccl, 4),
                "frac_of_roofline": round(ideal / ms_nccl, 3)})

    # ---- tensor-parallel decode consumer: 64 x 2560 partial rows all-reduced inside the kernel
    B, H = 64, 2560
    # two points, used alternately: a rank's slot of a point is rewritten only after every peer passed the other
    point_bytes = W * B * H * 8
    slots = SymmetricBuffer(2 * point_bytes, None, dev)
    it = [0]
    ep = torch.zeros(1, dtype=torch.int64, device=dev)
    x = torch.randn(B, 2048 // W, device=dev).to(torch.bfloat16)
    wgt = (torch.randn(H, 2048 // W, device=dev) * 0.02).to(torch.bfloat16)
    res = torch.randn(B, H, device=dev).to(torch.bfloat16)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    ws, meta = ops.gemm_partials(x, wgt)

    def tp_consumer():
        pt = it[0] % 2
        it[0] += 1
        ext().tp_step_begin(ep.data_ptr(), local)
        ext().dec_residual_norm_tp(ws, list(meta), res, nw, 1e-6, slots.ptrs, pt * point_bytes, B, ep.data_ptr(), r)

    ms = _timed(tp_consumer, iters=50)
    ops.check_errors(local)
    link_bytes = (W - 1) * B * H * 4   # the fp32 payload (the tags are protocol overhead)
    ideal = link_bytes / (LINK_GBS * 1e9) * 1e3
    out.append({"case": f"dec_residual_norm_tp_{B}x{H}", "world": W, "ms": round(ms, 4),
                "roofline_ms": round(ideal, 4), "frac_of_roofline": round(ideal / ms, 3),
                "note": "latency-bound: one one-way NVLink store per row, then the slowest rank"})
    red = torch.randn(B, H, device=dev)
    ms_nccl = _timed(lambda: dist.all_reduce(red), iters=50)
    out.append({"case": f"nccl_all_reduce_fp32_{B}x{H}", "world": W, "ms": round(ms_nccl, 4)})

    # ---- FSDP forward GEMM with the weight all-gathered inside the kernel (gate/up of the 4B model)
    M, N, K = 5112, 19456, 2560
    P = -(-N * K // (128 * W)) * 128 * W
    n_sh = P // W
    wsh = SymmetricBuffer(n_sh * 2, None, dev)
    wsh.view(0, (n_sh,), torch.bfloat16).copy_((torch.randn(n_sh, device=dev) * 0.02).to(torch.bfloat16))
    dst = torch.empty(P, dtype=torch.bfloat16, device=dev)
    flags = torch.zeros(4096, dtype=torch.int32, device=dev)
    ctr = torch.zeros(2, dtype=torch.int32, device=dev)
    sw = ops.ShardedWeight(dst[:N * K].view(N, K), wsh.ptrs, dst.data_ptr(), n_sh * 2, flags, ctr)
    x = (torch.randn(M, K, device=dev)).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    full = torch.empty(P, dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    dist.barrier()
    ms = _timed(lambda: ops.linear(x, sw, out=y), iters=10)
    ops.check_errors(local)
    y_fused = y.clone()
    link_bytes = (W - 1) * n_sh * 2
    flop_ms = 2.0 * M * N * K / (GEMM_TFLOPS * 1e12) * 1e3
    ideal = max(link_bytes / (LINK_GBS * 1e9) * 1e3, flop_ms)
    out.append({"case": f"gemm_gather_fwd_{M}x{K}x{N}", "world": W, "ms": round(ms, 4), "roofline_ms": round(ideal, 4),
                "gemm_only_roofline_ms": round(flop_ms, 4), "frac_of_roofline": round(ideal / ms, 3)})
    shard_local = wsh.view(0, (n_sh,), torch.bfloat16)

    def nccl_then_gemm():
        dist.all_gather_into_tensor(full, shard_local)
        ops.linear(x, full[:N * K].view(N, K), out=y)

    ms_nccl = _timed(nccl_then_gemm, iters=10)
    out.append({"case": f"nccl_all_gather_then_gemm_{M}x{K}x{N}", "world": W, "ms": round(ms_nccl, 4),
                "frac_of_roofline": round(ideal / ms_nccl, 3),
                "max_abs_diff_vs_fused": float((y.float() - y_fused.float()).abs().max())})
    ms_g = _timed(lambda: ops.linear(x, full[:N * K].view(N, K), out=y), iters=10)
    out.append({"case": f"gemm_only_{M}x{K}x{N}", "world": W, "ms": round(ms_g, 4)})
    # dgrad: dX [M, K] = dY [M, N] . W [N, K] (weight as the MN-major operand, gathered by k-blocks)
    dy = torch.randn(M, N, device=dev).to(torch.bfloat16)
    dx = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    ms = _timed(lambda: ops.grad_input(dy, sw, out=dx), iters=10)
    ops.check_errors(local)
    out.append({"case": f"gemm_gather_dgrad_{M}x{N}x{K}", "world": W, "ms": round(ms, 4), "roofline_ms": round(ideal, 4),
                "frac_of_roofline": round(ideal / ms, 3)})

    if r == 0:
        for row in out:
            print(json.dumps(row), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    for b in (grads, sig, params, slots, wsh):
        b.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
