// Skinny GEMM for the decode step: stream-K partial sums of x[M, K] . W[N, K]^T for M <= 64 rows.
//
// A decode-step GEMM reads every weight byte once and does at most 64 rows of math with it, so its time
// is the weight stream plus fixed per-launch costs.  This kernel keeps those costs small: no TMEM
// allocation or tensor-memory epilogue, a cp.async pipeline into 128-byte-swizzled shared memory,
// mma.sync m16n8k16 with fp32 accumulators in registers, and (while the weights are static, i.e. inside
// the decode loop) the first weight chunks requested before waiting for the previous kernel.
//
// Opt-in (VLMRL_SKINNY_GEMM=1).  Measured against the stream-K tcgen05 GEMM on the 4B decode shapes:
// faster alone for qkv / o_proj at batch 64 (20 vs 28 us, 15 vs 18 us, L2 evicted), slower for gate/up
// (35 vs 30 us), and slower in the graph-captured decode step (5.00 vs 3.92 ms), where the tcgen05
// kernel's early weight prefetch and programmatic launch overlap matter more.
//
// Work decomposition and output layout are exactly those of the stream-K tcgen05 GEMM (streamk.cuh): the
// U = tiles_n * kb_count (tile, 64-wide k-block) units are split evenly over the G CTAs, and each CTA
// writes one fp32 partial per tile segment to ws[slot][M][N].  So the decode consumers (dec_qkv,
// dec_residual_norm, dec_swiglu and the tensor-parallel consumer) read it unchanged.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"
#include "host_utils.h"
#include "mma_sync.cuh"
#include "streamk.cuh"
#include "vlm_ops.h"

namespace vlm {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kSkBN = 128;    // output columns per tile: 4 warps x 32
constexpr int kSkBK = 64;     // k-block
constexpr int kSkStages = 4;

// [rows][64] bf16 tile, 16-byte chunk c of row r stored at chunk c ^ (r & 7) (ldmatrix without conflicts)
VLM_DEV int sw64(int r, int col) { return r * 64 + ((((col >> 3) ^ (r & 7))) << 3) + (col & 7); }

template <int MT>
struct SkCfg {
  static constexpr int W_ELEMS = kSkBN * kSkBK;
  static constexpr int X_ELEMS = MT * 16 * kSkBK;
  static constexpr int SMEM = kSkStages * (W_ELEMS + X_ELEMS) * 2;
};

template <int MT>
__global__ void __launch_bounds__(128) skinny_partials_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                              const bf16* __restrict__ w, int64_t ldw,
                                                              float* __restrict__ ws, int M, int N, int K,
                                                              int kb_count, int64_t U, int prefetch_w) {
  using C = SkCfg<MT>;
  extern __shared__ __align__(128) uint8_t sk_smem[];
  bf16* sW = reinterpret_cast<bf16*>(sk_smem);
  bf16* sX = sW + kSkStages * C::W_ELEMS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const long long G = gridDim.x, c = blockIdx.x;
  const long long u_begin = c * U / G, u_end = (c + 1) * U / G;

  auto load_w = [&](int stage, int n0, int kb) {
    bf16* dst = sW + stage * C::W_ELEMS;
#pragma unroll
    for (int j = 0; j < kSkBN * 8 / 128; ++j) {
      const int i = tid + 128 * j, r = i >> 3, ch = i & 7;
      const int n = n0 + r, k = kb * kSkBK + ch * 8;
      const bool ok = n < N && k < K;
      cp_async16(dst + sw64(r, ch * 8), w + (ok ? static_cast<int64_t>(n) * ldw + k : 0), ok);
    }
  };
  auto load_x = [&](int stage, int kb) {
    bf16* dst = sX + stage * C::X_ELEMS;
#pragma unroll
    for (int j = 0; j < MT; ++j) {
      const int i = tid + 128 * j, r = i >> 3, ch = i & 7;
      const int k = kb * kSkBK + ch * 8;
      const bool ok = r < M && k < K;
      cp_async16(dst + sw64(r, ch * 8), x + (ok ? static_cast<int64_t>(r) * ldx + k : 0), ok);
    }
  };

  bool first_segment = true;
  for (long long u = u_begin; u < u_end;) {
    const int tile = static_cast<int>(u / kb_count);
    const int kb0 = static_cast<int>(u % kb_count);
    const int kb1 = static_cast<int>(min(static_cast<long long>(kb_count), kb0 + (u_end - u)));
    const int nkb = kb1 - kb0;
    const int n0 = tile * kSkBN;
    const long long first_unit = static_cast<long long>(tile) * kb_count;
    const int slot = static_cast<int>(c - ((first_unit + 1) * G - 1) / U);
    // prologue: STAGES-1 chunks in flight; the weight chunks of the first segment may go out before the
    // wait for the previous kernel (they are not written by it)
    if (first_segment && prefetch_w) {
      for (int s = 0; s < kSkStages - 1 && s < nkb; ++s) load_w(s, n0, kb0 + s);
      pdl_wait();
      pdl_trigger();
      for (int s = 0; s < kSkStages - 1; ++s) {
        if (s < nkb) load_x(s, kb0 + s);
        cp_async_commit();
      }
    } else {
      if (first_segment) {
        pdl_wait();
        pdl_trigger();
      }
      for (int s = 0; s < kSkStages - 1; ++s) {
        if (s < nkb) {
          load_w(s, n0, kb0 + s);
          load_x(s, kb0 + s);
        }
        cp_async_commit();
      }
    }
    first_segment = false;

    float acc[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) acc[mt][nb][0] = acc[mt][nb][1] = acc[mt][nb][2] = acc[mt][nb][3] = 0.f;

    for (int i = 0; i < nkb; ++i) {
      cp_async_wait<kSkStages - 2>();
      __syncthreads();
      const int st = i % kSkStages;
      const bf16* tw = sW + st * C::W_ELEMS;
      const bf16* tx = sX + st * C::X_ELEMS;
#pragma unroll
      for (int ks = 0; ks < kSkBK / 16; ++ks) {
        uint32_t a[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int r = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldsm_x4(a[mt], tx + sw64(r, ks * 16 + (lane >> 4) * 8));
        }
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b[4];
          const int r = warp * 32 + np * 16 + (lane & 7) + (lane >> 4) * 8;
          ldsm_x4(b, tw + sw64(r, ks * 16 + ((lane >> 3) & 1) * 8));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_bf16(acc[mt][2 * np], a[mt], b[0], b[1]);
            mma_bf16(acc[mt][2 * np + 1], a[mt], b[2], b[3]);
          }
        }
      }
      // the stage read STAGES-1 iterations from now was last read in iteration i-1 (all threads are past
      // this iteration's barrier), so it can be refilled
      const int nxt = i + kSkStages - 1;
      if (nxt < nkb) {
        load_w(nxt % kSkStages, n0, kb0 + nxt);
        load_x(nxt % kSkStages, kb0 + nxt);
      }
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();  // the next segment's prologue overwrites stages this one read

#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) {
        const int col = n0 + warp * 32 + nb * 8 + 2 * tq;
        if (col >= N) continue;
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        float* base = ws + static_cast<int64_t>(slot) * M * N;
        if (r0 < M)
          *reinterpret_cast<float2*>(base + static_cast<int64_t>(r0) * N + col) =
              make_float2(acc[mt][nb][0], acc[mt][nb][1]);
        if (r1 < M)
          *reinterpret_cast<float2*>(base + static_cast<int64_t>(r1) * N + col) =
              make_float2(acc[mt][nb][2], acc[mt][nb][3]);
      }
    }
    u += nkb;
  }
  if (u_begin >= u_end) {  // no work: still take part in the programmatic launch chain
    pdl_wait();
    pdl_trigger();
  }
}

template <int MT>
void launch_skinny(const at::Tensor& x, const at::Tensor& w, float* ws, int M, int N, int K, int kb_count, int64_t U,
                   int grid, bool prefetch_w) {
  auto kern = skinny_partials_kernel<MT>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SkCfg<MT>::SMEM));
    configured = true;
  }
  launch_pdl(kern, dim3(grid), dim3(128), SkCfg<MT>::SMEM, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const bf16*>(x.data_ptr()), static_cast<int64_t>(x.stride(0)),
             reinterpret_cast<const bf16*>(w.data_ptr()), static_cast<int64_t>(w.stride(0)), ws, M, N, K, kb_count, U,
             prefetch_w ? 1 : 0);
}

}  // namespace

bool skinny_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLMRL_SKINNY_GEMM");
    return e && e[0] == '1';
  }();
  return on;
}

// Partials of x . w^T for M <= 64 in the stream-K layout: (ws [slots, M, N] fp32, meta).
std::tuple<at::Tensor, std::vector<int64_t>> skinny_partials(const at::Tensor& x, const at::Tensor& w,
                                                             bool static_weights) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "skinny_partials: bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && x.size(1) == w.size(1),
              "skinny_partials: x [M, K], w [N, K] with contiguous rows");
  const int M = static_cast<int>(x.size(0)), N = static_cast<int>(w.size(0)), K = static_cast<int>(x.size(1));
  TORCH_CHECK(M >= 1 && M <= 64 && K % 8 == 0 && N % 8 == 0, "skinny_partials: M <= 64, K and N multiples of 8");
  TORCH_CHECK(x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "skinny_partials: 16-byte aligned rows");
  const c10::cuda::CUDAGuard g(x.device());
  const int tiles_n = (N + kSkBN - 1) / kSkBN, kb_count = (K + kSkBK - 1) / kSkBK;
  const int64_t U = static_cast<int64_t>(tiles_n) * kb_count;
  const int grid = static_cast<int>(std::min<int64_t>(U, num_sms(x.device().index())));
  const SkMeta m{M, N, 1, tiles_n, kb_count, grid, 128, kSkBN};
  // slots: at most the number of CTAs whose unit range meets one tile
  const int64_t per_cta = std::max<int64_t>(1, U / grid);
  const int64_t slots = std::min<int64_t>((kb_count + per_cta - 1) / per_cta + 1, grid);
  at::Tensor ws = at::empty({slots, M, N}, x.options().dtype(at::kFloat));
  float* wp = ws.data_ptr<float>();
  switch ((M + 15) / 16) {
    case 1: launch_skinny<1>(x, w, wp, M, N, K, kb_count, U, grid, static_weights); break;
    case 2: launch_skinny<2>(x, w, wp, M, N, K, kb_count, U, grid, static_weights); break;
    case 3: launch_skinny<3>(x, w, wp, M, N, K, kb_count, U, grid, static_weights); break;
    default: launch_skinny<4>(x, w, wp, M, N, K, kb_count, U, grid, static_weights); break;
  }
  return {ws, {m.M, m.N, m.tiles_m, m.tiles_n, m.kb_count, m.grid, m.bm, m.bn}};
}

}  // namespace vlm
