// Peer-memory collectives over NVLink / NVSwitch for the FSDP engine (one process per GPU).
//
// Every rank allocates its buffers with cudaMalloc, exports them as CUDA IPC handles and maps the
// peers' buffers into its own address space (the handles travel over the process group), so a
// kernel can load from and store to any rank's memory directly.  Three kernels use that:
//
//  * rs_pull_kernel      gradient reduce-scatter: after signalling "my full-unit fp32 gradient is
//                        complete" to every peer and waiting for theirs, each rank reads ITS shard
//                        of every rank's gradient over NVLink, sums in rank order and accumulates
//                        into its local fp32 gradient shard (RS fused with the accumulate).
//  * adamw_push_kernel   sharded AdamW fused with the parameter all-gather: the updated fp32 shard
//                        is rounded to bf16 and stored straight into the gathered bf16 unit of EVERY
//                        rank (peer stores), then each CTA publishes a release-increment on every
//                        peer's arrival counter.
//  * peer_wait_kernel    waits until every peer's push CTAs have arrived (bounded), so the gathered
//                        buffers are complete before the next forward reads them.
//
// Signalling uses 64-bit monotonic counters in an IPC-shared signal pad: slot s holds one counter
// per source rank; writers publish with st/red.release.sys, readers poll with ld.acquire.sys.
// Epochs never reset, so no slot needs clearing between uses.  Every wait is bounded (kPeerWait
// cycles): on timeout the kernel records kErrTimeoutPeer in the device error word and returns
// without touching data; the host raises when it reads the word.
//
// No reference counterpart: the reference has no explicit collectives (its FSDP plan in
// utils/sharding.py:23-48 would leave them to XLA).

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"

namespace vlm {

using bf16 = __nv_bfloat16;

// Wait until sig[slot * W + p] >= target for every peer p != rank.  Called by one thread.
VLM_DEV bool wait_peers(const unsigned long long* sig, int slot, int W, int rank, unsigned long long target,
                        int* err) {
  return wait_peers_at(sig, static_cast<int64_t>(slot) * W, W, rank, target, err);
}

// ------------------------------------------------------------------ reduce-scatter (pull)
// WR = number of ranks (compile time), so every rank's loads of a vector group are issued together and
// the NVLink and local HBM latencies overlap; the sum is still taken in rank order.
template <int WR>
__global__ void __launch_bounds__(256) rs_pull_kernel(PeerTable bufs, int64_t shard_off, int64_t n, float* out,
                                                      int accumulate, PeerTable sigs, int slot,
                                                      unsigned long long epoch, int rank, int* err) {
  constexpr int W = WR;
  __shared__ int ok;
  if (blockIdx.x == 0 && threadIdx.x < W && static_cast<int>(threadIdx.x) != rank) {
    __threadfence_system();
    store_release_sys(reinterpret_cast<unsigned long long*>(sigs.p[threadIdx.x]) + static_cast<int64_t>(slot) * W + rank,
                      epoch);
  }
  if (threadIdx.x == 0)
    ok = wait_peers(reinterpret_cast<const unsigned long long*>(sigs.p[rank]), slot, W, rank, epoch, err);
  __syncthreads();
  if (!ok) return;
  // U float4 per rank in flight per thread: W * U * 16 bytes
  constexpr int U = W <= 4 ? 4 : 2;
  const int64_t n4 = n >> 2;
  float4* o4 = reinterpret_cast<float4*>(out);
  const float4* src[W];
#pragma unroll
  for (int q = 0; q < W; ++q) src[q] = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(bufs.p[q]) + shard_off);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < n4; base += stride * U) {
    float4 x[W][U];
    float4 acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * stride;
      acc[u] = (accumulate && i < n4) ? o4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < W; ++q) x[q][u] = i < n4 ? __ldcg(src[q] + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int q = 0; q < W; ++q) {
        acc[u].x += x[q][u].x;
        acc[u].y += x[q][u].y;
        acc[u].z += x[q][u].z;
        acc[u].w += x[q][u].w;
      }
      const int64_t i = base + u * stride;
      if (i < n4) o4[i] = acc[u];
    }
  }
}

// ------------------------------------------------------------------ AdamW + all-gather (push)
__global__ void __launch_bounds__(256) adamw_push_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                         float* __restrict__ m, float* __restrict__ v, PeerTable dst,
                                                         int64_t dst_off, int64_t n, const float* __restrict__ scale_ptr,
                                                         float lr, float b1, float b2, float eps, float wd, float bc1,
                                                         float bc2, PeerTable sigs, int slot, int rank, int W) {
  const float scale = *scale_ptr;
  const int64_t n8 = n >> 3;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float pv[8], gv[8], mv[8], vv[8];
    *reinterpret_cast<float4*>(pv) = reinterpret_cast<const float4*>(p)[2 * i];
    *reinterpret_cast<float4*>(pv + 4) = reinterpret_cast<const float4*>(p)[2 * i + 1];
    *reinterpret_cast<float4*>(gv) = reinterpret_cast<const float4*>(g)[2 * i];
    *reinterpret_cast<float4*>(gv + 4) = reinterpret_cast<const float4*>(g)[2 * i + 1];
    *reinterpret_cast<float4*>(mv) = reinterpret_cast<const float4*>(m)[2 * i];
    *reinterpret_cast<float4*>(mv + 4) = reinterpret_cast<const float4*>(m)[2 * i + 1];
    *reinterpret_cast<float4*>(vv) = reinterpret_cast<const float4*>(v)[2 * i];
    *reinterpret_cast<float4*>(vv + 4) = reinterpret_cast<const float4*>(v)[2 * i + 1];
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gi = gv[j] * scale;
      mv[j] = b1 * mv[j] + (1.f - b1) * gi;
      vv[j] = b2 * vv[j] + (1.f - b2) * gi * gi;
      const float upd = (mv[j] / bc1) / (sqrtf(vv[j] / bc2) + eps) + wd * pv[j];
      pv[j] = pv[j] - lr * upd;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) packed[j] = pack_bf16x2(pv[2 * j], pv[2 * j + 1]);
    reinterpret_cast<float4*>(p)[2 * i] = *reinterpret_cast<float4*>(pv);
    reinterpret_cast<float4*>(p)[2 * i + 1] = *reinterpret_cast<float4*>(pv + 4);
    reinterpret_cast<float4*>(m)[2 * i] = *reinterpret_cast<float4*>(mv);
    reinterpret_cast<float4*>(m)[2 * i + 1] = *reinterpret_cast<float4*>(mv + 4);
    reinterpret_cast<float4*>(v)[2 * i] = *reinterpret_cast<float4*>(vv);
    reinterpret_cast<float4*>(v)[2 * i + 1] = *reinterpret_cast<float4*>(vv + 4);
    const uint4 val = make_uint4(packed[0], packed[1], packed[2], packed[3]);
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < W) reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(dst.p[q]) + dst_off)[i] = val;
  }
  // publish: every thread's peer stores are ordered before the CTA's arrival increments
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W && static_cast<int>(threadIdx.x) != rank)
    add_release_sys(reinterpret_cast<unsigned long long*>(sigs.p[threadIdx.x]) + static_cast<int64_t>(slot) * W + rank,
                    1ull);
}

__global__ void peer_wait_kernel(const unsigned long long* sig, int slot, unsigned long long target, int rank, int W,
                                 int* err, long long budget) {
  if (threadIdx.x == 0) wait_peers_at(sig, static_cast<int64_t>(slot) * W, W, rank, target, err, budget);
}

// Every rank signals slot `slot` with `epoch` and waits for all peers to reach it (a device-side barrier).
__global__ void peer_barrier_kernel(PeerTable sigs, int slot, unsigned long long epoch, int rank, int W, int* err) {
  if (threadIdx.x < W && static_cast<int>(threadIdx.x) != rank) {
    __threadfence_system();
    store_release_sys(reinterpret_cast<unsigned long long*>(sigs.p[threadIdx.x]) + static_cast<int64_t>(slot) * W + rank,
                      epoch);
  }
  __syncthreads();
  if (threadIdx.x == 0) wait_peers(reinterpret_cast<const unsigned long long*>(sigs.p[rank]), slot, W, rank, epoch, err);
}

// ------------------------------------------------------------------ host: IPC-shared allocations
int64_t symm_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  VLM_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  VLM_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  VLM_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

at::Tensor symm_ipc_handle(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  VLM_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  at::Tensor out = at::empty({static_cast<int64_t>(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t symm_open(at::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)) && handle.scalar_type() == at::kByte,
              "symm_open: expected a ", sizeof(cudaIpcMemHandle_t), "-byte handle");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  VLM_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  VLM_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// Non-owning tensor over bytes [offset, offset + numel * itemsize) of an allocation.
at::Tensor symm_view(int64_t base, int64_t offset_bytes, std::vector<int64_t> sizes, at::ScalarType dtype,
                     int64_t device) {
  return torch::from_blob(reinterpret_cast<char*>(base) + offset_bytes, sizes,
                          at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
}

static PeerTable make_table(const std::vector<int64_t>& ptrs, int64_t byte_off = 0) {
  return make_peer_table(ptrs, byte_off);
}

static int peer_grid(int64_t items, int device) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, num_sms(device) * 2)));
}

// out (+)= sum over ranks q of unit_q[shard_off : shard_off + n]; unit_q = bufs[q] + unit_off bytes.
void rs_pull(std::vector<int64_t> bufs, int64_t unit_off_bytes, int64_t shard_off, at::Tensor out, bool accumulate,
             std::vector<int64_t> sigs, int64_t slot, int64_t epoch, int64_t rank, int64_t max_ctas) {
  const int W = static_cast<int>(bufs.size());
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() % 4 == 0, "rs_pull: fp32 x4");
  TORCH_CHECK(static_cast<int>(sigs.size()) == W && rank >= 0 && rank < W, "rs_pull: tables");
  TORCH_CHECK((unit_off_bytes + shard_off * 4) % 16 == 0, "rs_pull: 16-byte aligned shards");
  const c10::cuda::CUDAGuard g(out.device());
  const int dev = out.device().index();
  // two 256-thread CTAs per SM by default: they fit beside a GEMM CTA of the backward they overlap (no
  // shared memory, 512 threads), and at 2 GPUs they pulled 617 GB/s against 526 GB/s with one per SM;
  // max_ctas > 0 sets the grid explicitly
  const int64_t want = max_ctas > 0 ? max_ctas : 2 * num_sms(dev);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((out.numel() / 4 + 255) / 256, want)));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const PeerTable tb = make_table(bufs, unit_off_bytes), ts = make_table(sigs);
  float* o = out.data_ptr<float>();
  const int acc = accumulate ? 1 : 0, sl = static_cast<int>(slot), rk = static_cast<int>(rank);
  const auto ep = static_cast<unsigned long long>(epoch);
  switch (W) {
    case 1: rs_pull_kernel<1><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 2: rs_pull_kernel<2><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 3: rs_pull_kernel<3><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 4: rs_pull_kernel<4><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 5: rs_pull_kernel<5><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 6: rs_pull_kernel<6><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    case 7: rs_pull_kernel<7><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
    default: rs_pull_kernel<8><<<grid, 256, 0, st>>>(tb, shard_off, out.numel(), o, acc, ts, sl, ep, rk, err_word(dev)); break;
  }
  VLM_LAUNCHED();
}

// AdamW on this rank's shard; the bf16 result is stored at dst[q] + dst_off_bytes for every rank q.
// Returns the number of CTAs launched (each adds 1 to every peer's counter in `slot`).
int64_t adamw_push(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, std::vector<int64_t> dst,
                   int64_t dst_off_bytes, at::Tensor scale, double lr, double b1, double b2, double eps, double wd,
                   int64_t step, std::vector<int64_t> sigs, int64_t slot, int64_t rank) {
  const int W = static_cast<int>(dst.size());
  const int64_t n = p.numel();
  TORCH_CHECK(n % 8 == 0 && p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
              "adamw_push: contiguous fp32 shards of a multiple of 8 elements");
  TORCH_CHECK(dst_off_bytes % 16 == 0, "adamw_push: 16-byte aligned destination");
  TORCH_CHECK(static_cast<int>(sigs.size()) == W, "adamw_push: tables");
  const c10::cuda::CUDAGuard gd(p.device());
  const int dev = p.device().index();
  const float bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  const float bc2 = static_cast<float>(1.0 - std::pow(b2, static_cast<double>(step)));
  const int grid = peer_grid(n / 8, dev);
  adamw_push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), make_table(dst, dst_off_bytes),
      0, n, scale.data_ptr<float>(), static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2),
      static_cast<float>(eps), static_cast<float>(wd), bc1, bc2, make_table(sigs), static_cast<int>(slot),
      static_cast<int>(rank), W);
  VLM_LAUNCHED();
  return grid;
}

// budget_cycles <= 0 selects the default (kPeerWait); tests pass a short budget to exercise the timeout.
void peer_wait(int64_t local_sig, int64_t slot, int64_t target, int64_t rank, int64_t world, int64_t device,
               int64_t budget_cycles) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  peer_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const unsigned long long*>(local_sig), static_cast<int>(slot),
      static_cast<unsigned long long>(target), static_cast<int>(rank), static_cast<int>(world),
      err_word(static_cast<int>(device)), budget_cycles > 0 ? budget_cycles : kPeerWait);
  VLM_LAUNCHED();
}

void peer_barrier(std::vector<int64_t> sigs, int64_t slot, int64_t epoch, int64_t rank, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  peer_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(sigs), static_cast<int>(slot), static_cast<unsigned long long>(epoch), static_cast<int>(rank),
      static_cast<int>(sigs.size()), err_word(static_cast<int>(device)));
  VLM_LAUNCHED();
}

}  // namespace vlm
