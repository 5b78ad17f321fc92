// Flash-attention forward on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
// Varlen (cu_seqlens) GQA attention, causal or not, with an optional shared prefix per segment
// (pre[b] = (start, len): keys every query of segment b also sees, without the causal mask).  Same
// contract as flash_fwd_kernel in attention.cu, which stays the path for head dims other than 64/128.
//
// One CTA = 128 query rows of one head of one segment; 4 warps, thread r owns row r (TMEM lane r).
// Per 64-key block j:
//   thread 0   S = Q . K_j^T            tcgen05.mma kind::f16, 128 x 64 x D, fp32 accumulator in TMEM
//   all        tcgen05.ld the row of S, scale + mask, online softmax (running max m, sum l) in registers
//   all        P (bf16) -> shared memory in the 128-byte-swizzled K-major layout the MMA reads;
//              O (TMEM) rescaled by exp2(m_old - m_new) with tcgen05.ld/st, only in warps whose max moved
//   thread 0   O += P . V_j             tcgen05.mma 128 x D x 64 (V is the MN-major operand)
// Q, K and V are staged by TMA with 128-byte swizzle; K is double buffered and V(j) is loaded while the
// softmax of block j runs.  Every wait is bounded: on timeout the kernel records kErrTimeoutFlag, drains
// its own MMAs and copies, frees TMEM and returns.
//
// Reference counterpart: the XLA lowering of the attention in models/qwen3vl/model.py:523-578 (text) and
// vision.py:45-113 (ViT).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"
#include "host_utils.h"
#include "vlm_ops.h"

namespace vlm {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kBM = 128;  // query rows per CTA
constexpr int kBN = 64;   // keys per block
constexpr float kLog2eTc = 1.4426950408889634f;
constexpr float kLn2Tc = 0.6931471805599453f;

template <int D>
struct TcCfg {
  static constexpr int Q_BYTES = kBM * D * 2;   // D/64 sub-tiles [128 rows][128 B]
  static constexpr int KV_BYTES = kBN * D * 2;  // D/64 sub-tiles [64 rows][128 B]
  static constexpr int P_BYTES = kBM * kBN * 2; // [128 rows][128 B]
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_BYTES;                      // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;         // 1 stage
  static constexpr int P_OFF = V_OFF + KV_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 128;
  // S (64 columns) then O (D columns).  Shared memory admits 4 CTAs per SM at D = 64 and 2 at D = 128, so
  // 128 / 256 columns keep their sum within the SM's 512 TMEM columns.
  static constexpr uint32_t S_COL = 0, O_COL = D == 64 ? 64 : 128, TMEM_COLS = D == 64 ? 128 : 256;
};

VLM_DEV void fence_proxy_async_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                           const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV,
                                                           const int* __restrict__ cu, bf16* __restrict__ O,
                                                           float* __restrict__ LSE, int Hq, int Hkv, int T,
                                                           float scale_log2, const int* __restrict__ pre, int* err) {
  using C = TcCfg<D>;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = cu[b], L = cu[b + 1] - s0;
  const int q0 = qt * kBM;
  if (q0 >= L) return;
  const int pstart = pre ? pre[2 * b] : 0, plen = pre ? pre[2 * b + 1] : 0;
  const int hk = h / (Hq / Hkv);
  const int nkp = (plen + kBN - 1) / kBN;
  const int nko = CAUSAL ? min((L + kBN - 1) / kBN, (q0 + kBM) / kBN) : (L + kBN - 1) / kBN;
  const int nkb = nkp + nko;

  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + C::Q_OFF;
  uint8_t* sK = sm + C::K_OFF;
  uint8_t* sV = sm + C::V_OFF;
  uint8_t* sP = sm + C::P_OFF;
  uint64_t* qbar = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* kfull = qbar + 1;  // [2]
  uint64_t* vfull = qbar + 3;
  uint64_t* sbar = qbar + 4;
  uint64_t* pvbar = qbar + 5;
  uint64_t* drain = qbar + 6;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(qbar + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  // key block j -> (first key row in the K/V tensors, first key index for masking, key limit, causal?)
  auto key_row = [&](int j) { return j < nkp ? pstart + j * kBN : s0 + (j - nkp) * kBN; };

  auto load_kv = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bar, int j) {
    mbar_arrive_expect_tx(bar, C::KV_BYTES);
#pragma unroll
    for (int c = 0; c < D / 64; ++c) tma_load_2d(dst + c * (kBN * 128), map, bar, hk * D + 64 * c, key_row(j));
  };

  if (tid == 0) {
    mbar_init(qbar, 1);
    mbar_init(&kfull[0], 1);
    mbar_init(&kfull[1], 1);
    mbar_init(vfull, 1);
    mbar_init(sbar, 1);
    mbar_init(pvbar, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  pdl_wait();
  int k_issued = 0, v_issued = 0;
  if (tid == 0) {
    mbar_arrive_expect_tx(qbar, C::Q_BYTES);
#pragma unroll
    for (int c = 0; c < D / 64; ++c) tma_load_2d(sQ + c * (kBM * 128), &tmQ, qbar, h * D + 64 * c, s0 + q0);
    load_kv(&tmK, sK, &kfull[0], 0);
    load_kv(&tmV, sV, vfull, 0);
    k_issued = v_issued = 1;
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV), sPa = smem_u32(sP);
  constexpr uint32_t idesc_s = idesc_bf16_f32(kBM, kBN, false, false);
  constexpr uint32_t idesc_o = idesc_bf16_f32(kBM, D, false, true);

  const int r = tid;          // row of this thread in the tile
  const int qi = q0 + r;      // query index inside the segment
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int j = 0; j < nkb && ok; ++j) {
    // ---- thread 0: S(j), K(j+1), V(j)
    if (tid == 0) {
      bool t_ok = true;
      if (j == 0) t_ok = mbar_wait(qbar, 0, abort_flag, err, kErrTimeoutFlag);
      t_ok = t_ok && mbar_wait(&kfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, err, kErrTimeoutFlag);
      if (t_ok) {
        tc_fence_after();
        const uint32_t kst = sKa + (j & 1) * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(sQa + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(kst + (kk >> 2) * (kBN * 128) + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + C::S_COL, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(sbar);
        if (j + 1 < nkb) {  // stage (j+1)&1 was last read by S(j-1), which every thread has waited for
          load_kv(&tmK, sK + ((j + 1) & 1) * C::KV_BYTES, &kfull[(j + 1) & 1], j + 1);
          ++k_issued;
        }
        if (j > 0) {  // V(j) may overwrite V(j-1) once PV(j-1) is done
          t_ok = mbar_wait(pvbar, static_cast<uint32_t>((j - 1) & 1), abort_flag, err, kErrTimeoutFlag);
          if (t_ok) {
            load_kv(&tmV, sV, vfull, j);
            ++v_issued;
          }
        }
      }
      if (!t_ok) *abort_flag = 1;
    }
    // ---- all: softmax of the S row
    ok = mbar_wait(sbar, static_cast<uint32_t>(j & 1), abort_flag, err, kErrTimeoutFlag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t sr[kBN / 16][16];
#pragma unroll
    for (int c = 0; c < kBN / 16; ++c) tmem_ld16(tmem + lane_base + C::S_COL + 16 * c, sr[c]);
    tmem_ld_wait();
    const bool in_pre = j < nkp;
    const int key0 = in_pre ? j * kBN : (j - nkp) * kBN;
    const int klim = in_pre ? plen : L;
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < kBN / 16; ++c) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int key = key0 + 16 * c + e;
        const bool valid = key < klim && (!CAUSAL || in_pre || key <= qi);
        const float v = valid ? __uint_as_float(sr[c][e]) * scale_log2 : -INFINITY;
        sr[c][e] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
    }
    const float m_new = fmaxf(m_run, mx);
    const float base = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = exp2f(m_run - base);
    float psum = 0.f;
    uint32_t pk[kBN / 2];
#pragma unroll
    for (int c = 0; c < kBN / 16; ++c) {
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const float p0 = exp2f(__uint_as_float(sr[c][e]) - base);
        const float p1 = exp2f(__uint_as_float(sr[c][e + 1]) - base);
        psum += p0 + p1;
        pk[(16 * c + e) / 2] = pack_bf16x2(p0, p1);
      }
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
    // ---- all: P(j) -> shared memory and O rescale, once PV(j-1) no longer reads sP / writes O
    if (j > 0) {
      ok = mbar_wait(pvbar, static_cast<uint32_t>((j - 1) & 1), abort_flag, err, kErrTimeoutFlag);
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
    }
#pragma unroll
    for (int ch = 0; ch < kBN / 8; ++ch)
      *reinterpret_cast<uint4*>(sP + r * 128 + ((ch ^ (r & 7)) << 4)) =
          make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
    if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 64) {
        uint32_t o[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld16(tmem + lane_base + C::O_COL + c0 + 16 * c, o[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c][e] = __float_as_uint(__uint_as_float(o[c][e]) * alpha);
          tmem_st16(tmem + lane_base + C::O_COL + c0 + 16 * c, o[c]);
        }
      }
      tmem_st_wait();
    }
    fence_proxy_async_cta();
    tc_fence_before();
    __syncthreads();
    // ---- thread 0: O += P(j) . V(j)
    if (tid == 0) {
      tc_fence_after();
      if (mbar_wait(vfull, static_cast<uint32_t>(j & 1), abort_flag, err, kErrTimeoutFlag)) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(sPa + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sVa + kk * 2048, 8192, 1024);
          umma_f16(tmem + C::O_COL, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pvbar);
      } else {
        *abort_flag = 1;
      }
    }
  }

  if (ok && nkb > 0) {
    ok = mbar_wait(pvbar, static_cast<uint32_t>((nkb - 1) & 1), abort_flag, err, kErrTimeoutFlag);
    ok = !__syncthreads_or(!ok);
  }
  if (ok && nkb > 0) {
    tc_fence_after();
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    const bool row_ok = qi < L;
    bf16* orow = O + (static_cast<int64_t>(s0 + qi) * Hq + h) * D;
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 64) {
      uint32_t o[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16(tmem + lane_base + C::O_COL + c0 + 16 * c, o[c]);
      tmem_ld_wait();
      if (row_ok) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w[e] = pack_bf16x2(__uint_as_float(o[c][2 * e]) * inv, __uint_as_float(o[c][2 * e + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + c0 + 16 * c);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
    if (row_ok) LSE[static_cast<int64_t>(h) * T + s0 + qi] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2Tc : -INFINITY;
  }
  if (!ok && tid == 0) {
    // drain: every MMA this thread issued, then every copy still in flight (bounded waits)
    volatile int no_abort = 0;
    umma_commit(drain);
    mbar_wait(drain, 0, &no_abort, nullptr, 0);
    if (k_issued > 0) {
      // K(k_issued-1) is the newest copy; the older one (if any) was consumed or is waited on as well
      for (int i = max(0, k_issued - 2); i < k_issued; ++i)
        mbar_wait(&kfull[i & 1], static_cast<uint32_t>((i >> 1) & 1), &no_abort, nullptr, 0);
    }
    if (v_issued > 0) mbar_wait(vfull, static_cast<uint32_t>((v_issued - 1) & 1), &no_abort, nullptr, 0);
    mbar_wait(qbar, 0, &no_abort, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, bool CAUSAL>
void launch_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu, at::Tensor& o,
               at::Tensor& lse, int max_seqlen, float scale, const int* pre) {
  using C = TcCfg<D>;
  const int B = static_cast<int>(cu.numel() - 1), Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(k.size(1));
  const int T = static_cast<int>(q.size(0));
  const CUtensorMap tq = make_tmap_2d_bf16(q.data_ptr(), static_cast<int64_t>(Hq) * D, T, static_cast<int64_t>(Hq) * D,
                                           64, kBM);
  const CUtensorMap tk = make_tmap_2d_bf16(k.data_ptr(), static_cast<int64_t>(Hkv) * D, T,
                                           static_cast<int64_t>(Hkv) * D, 64, kBN);
  const CUtensorMap tv = make_tmap_2d_bf16(v.data_ptr(), static_cast<int64_t>(Hkv) * D, T,
                                           static_cast<int64_t>(Hkv) * D, 64, kBN);
  auto kern = flash_fwd_tc_kernel<D, CAUSAL>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  const dim3 grid((max_seqlen + kBM - 1) / kBM, Hq, B);
  launch_pdl(kern, grid, dim3(128), C::SMEM, at::cuda::getCurrentCUDAStream(), tq, tk, tv, cu.data_ptr<int>(),
             reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), Hq, Hkv, T, scale * kLog2eTc, pre,
             err_word(q.device().index()));
}


// ------------------------------------------------------------------ backward: dK, dV
// One CTA = 128 keys of one KV head of one segment; 4 warps, thread r owns key row r (TMEM lane r).  For
// each of the rep query heads sharing the KV head and each 64-query chunk that sees these keys (the
// segment's own queries at or after the keys, causal; then xq = the member queries of segments that use
// this one as a shared prefix, unmasked):
//   thread 0   S^T = K . Q^T and dP^T = V . dO^T       tcgen05.mma 128 x 64 x D into TMEM
//   all        P = exp2(S^T * scale_log2 - lse_log2), dS = P * (dP - delta), both bf16 into shared memory
//   thread 0   dV += P^T . dO and dK += dS^T . Q        tcgen05.mma 128 x D x 64 (Q and dO chunks read as the
//                                                      MN-major operand: the same tiles as above)
// dK is scaled once at the end.  The Q / dO chunks are TMA-staged in two buffers; LSE and delta of the next
// chunk are read while the current one's MMAs run.  Every wait is bounded (as in the forward).
template <int D>
struct TcBwdCfg {
  static constexpr int K_BYTES = kBM * D * 2;    // D/64 sub-tiles [128 rows][128 B]
  static constexpr int C_BYTES = 64 * D * 2;     // a 64-query chunk: D/64 sub-tiles [64 rows][128 B]
  static constexpr int P_BYTES = kBM * 64 * 2;   // [128 rows][128 B]
  static constexpr int K_OFF = 0, V_OFF = K_BYTES;
  static constexpr int Q_OFF = 2 * K_BYTES;                 // [2] chunks
  static constexpr int DO_OFF = Q_OFF + 2 * C_BYTES;        // [2] chunks
  static constexpr int P_OFF = DO_OFF + 2 * C_BYTES;
  static constexpr int DS_OFF = P_OFF + P_BYTES;
  static constexpr int L_OFF = DS_OFF + P_BYTES;            // float [2][64] lse (log2 units), [2][64] delta
  static constexpr int BAR_OFF = L_OFF + 4 * 64 * 4;
  static constexpr int SMEM = 1024 + BAR_OFF + 128;
  static constexpr uint32_t ST_COL = 0, DP_COL = 64, DV_COL = 128, DK_COL = D == 64 ? 192 : 256;
  static constexpr uint32_t TMEM_COLS = D == 64 ? 256 : 512;
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_bwd_dkdv_tc_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, const float* __restrict__ LSE,
    const float* __restrict__ DELTA, const int* __restrict__ cu, bf16* __restrict__ dK, bf16* __restrict__ dV, int Hq,
    int Hkv, int T, float scale_log2, float scale, const int* __restrict__ xq, int* err) {
  using C = TcBwdCfg<D>;
  const int kblk = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int s0 = cu[b], L = cu[b + 1] - s0;
  const int k0 = kblk * kBM;
  if (k0 >= L) return;
  const int xs = xq ? xq[2 * b] : 0, xlen = xq ? xq[2 * b + 1] - xq[2 * b] : 0;
  const int rep = Hq / Hkv;
  const int qc_start = CAUSAL ? k0 / 64 : 0;
  const int n_own = (L + 63) / 64 - qc_start;
  const int n_chunks = n_own + (xlen + 63) / 64;
  const int total = rep * n_chunks;

  extern __shared__ __align__(1024) uint8_t tcb_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tcb_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm + C::K_OFF;
  uint8_t* sV = sm + C::V_OFF;
  uint8_t* sQ = sm + C::Q_OFF;
  uint8_t* sdO = sm + C::DO_OFF;
  uint8_t* sP = sm + C::P_OFF;
  uint8_t* sdS = sm + C::DS_OFF;
  float* sL = reinterpret_cast<float*>(sm + C::L_OFF);  // [2][64]
  float* sDl = sL + 2 * 64;                              // [2][64]
  uint64_t* kvbar = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* qfull = kvbar + 1;  // [2]
  uint64_t* sbar = kvbar + 3;
  uint64_t* gbar = kvbar + 4;
  uint64_t* drain = kvbar + 5;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(kvbar + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int tid = threadIdx.x, warp = tid >> 5;

  // chunk it -> (query head, first query row in the tensors, first query index inside its range, limit, own?)
  struct Chunk {
    int hh, row0, qs, qlim;
    bool own;
  };
  auto chunk = [&](int it) {
    Chunk ch;
    ch.hh = hk * rep + it / n_chunks;
    const int c = it % n_chunks;
    ch.own = c < n_own;
    ch.qs = ch.own ? (qc_start + c) * 64 : (c - n_own) * 64;
    ch.qlim = ch.own ? L : xlen;
    ch.row0 = (ch.own ? s0 : xs) + ch.qs;
    return ch;
  };
  auto load_chunk = [&](int it) {
    const Chunk ch = chunk(it);
    uint64_t* bar = &qfull[it & 1];
    mbar_arrive_expect_tx(bar, 2 * C::C_BYTES);
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      tma_load_2d(sQ + (it & 1) * C::C_BYTES + c * (64 * 128), &tmQ, bar, ch.hh * D + 64 * c, ch.row0);
      tma_load_2d(sdO + (it & 1) * C::C_BYTES + c * (64 * 128), &tmdO, bar, ch.hh * D + 64 * c, ch.row0);
    }
  };
  auto load_stats = [&](int it) {  // LSE (log2 units) and delta of chunk it; +inf LSE masks a query
    if (tid < 64) {
      const Chunk ch = chunk(it);
      const bool ok = ch.qs + tid < ch.qlim;
      const int64_t idx = static_cast<int64_t>(ch.hh) * T + ch.row0 + tid;
      sL[(it & 1) * 64 + tid] = ok ? LSE[idx] * kLog2eTc : INFINITY;
      sDl[(it & 1) * 64 + tid] = ok ? DELTA[idx] : 0.f;
    }
  };

  if (tid == 0) {
    mbar_init(kvbar, 1);
    mbar_init(&qfull[0], 1);
    mbar_init(&qfull[1], 1);
    mbar_init(sbar, 1);
    mbar_init(gbar, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  pdl_wait();
  if (tid == 0 && total > 0) {
    mbar_arrive_expect_tx(kvbar, 2 * C::K_BYTES);
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      tma_load_2d(sK + c * (kBM * 128), &tmK, kvbar, hk * D + 64 * c, s0 + k0);
      tma_load_2d(sV + c * (kBM * 128), &tmV, kvbar, hk * D + 64 * c, s0 + k0);
    }
    load_chunk(0);
    if (total > 1) load_chunk(1);
  }
  if (total > 0) load_stats(0);
  if (warp == 0) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t sKa = smem_u32(sK), sVa = smem_u32(sV), sQa = smem_u32(sQ), sdOa = smem_u32(sdO);
  const uint32_t sPa = smem_u32(sP), sdSa = smem_u32(sdS);
  constexpr uint32_t idesc_s = idesc_bf16_f32(kBM, 64, false, false);
  constexpr uint32_t idesc_g = idesc_bf16_f32(kBM, D, false, true);
  const int r = tid, key = k0 + r;  // key index inside the segment
  bool ok = true;
  int loads_issued = total > 1 ? 2 : total;

  for (int it = 0; it < total && ok; ++it) {
    const int st = it & 1;
    const Chunk ch = chunk(it);
    if (tid == 0) {
      bool t_ok = it > 0 || mbar_wait(kvbar, 0, abort_flag, err, kErrTimeoutFlag);
      t_ok = t_ok && mbar_wait(&qfull[st], static_cast<uint32_t>((it >> 1) & 1), abort_flag, err, kErrTimeoutFlag);
      if (t_ok) {
        tc_fence_after();
        const uint32_t qa = sQa + st * C::C_BYTES, da = sdOa + st * C::C_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * (kBM * 128) + (kk & 3) * 32, co = (kk >> 2) * (64 * 128) + (kk & 3) * 32;
          umma_f16(tmem + C::ST_COL, sdesc_sw128(sKa + ko, 16, 1024), sdesc_sw128(qa + co, 16, 1024), idesc_s,
                   kk > 0 ? 1u : 0u);
          umma_f16(tmem + C::DP_COL, sdesc_sw128(sVa + ko, 16, 1024), sdesc_sw128(da + co, 16, 1024), idesc_s,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(sbar);
      } else {
        *abort_flag = 1;
      }
    }
    ok = mbar_wait(sbar, static_cast<uint32_t>(it & 1), abort_flag, err, kErrTimeoutFlag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t sv[4][16], dp[4][16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      tmem_ld16(tmem + lane_base + C::ST_COL + 16 * c, sv[c]);
      tmem_ld16(tmem + lane_base + C::DP_COL + 16 * c, dp[c]);
    }
    tmem_ld_wait();
    uint32_t pk[32], dk2[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        float pr[2], ds[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int q = 16 * c + e + h;
          const bool valid = key < L && (!CAUSAL || !ch.own || key <= ch.qs + q);
          const float pv = valid ? exp2f(__uint_as_float(sv[c][e + h]) * scale_log2 - sL[st * 64 + q]) : 0.f;
          pr[h] = pv;
          ds[h] = pv * (__uint_as_float(dp[c][e + h]) - sDl[st * 64 + q]);
        }
        pk[(16 * c + e) / 2] = pack_bf16x2(pr[0], pr[1]);
        dk2[(16 * c + e) / 2] = pack_bf16x2(ds[0], ds[1]);
      }
    }
    // the previous chunk's dV / dK MMAs read sP / sdS: wait for them before overwriting
    if (it > 0) {
      ok = mbar_wait(gbar, static_cast<uint32_t>((it - 1) & 1), abort_flag, err, kErrTimeoutFlag);
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      // chunk it+1 goes into the buffers chunk it-1 used, now that its dV / dK MMAs are done
      if (tid == 0 && it + 1 < total && it + 1 >= 2) {
        load_chunk(it + 1);
        ++loads_issued;
      }
    }
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      const int off = r * 128 + ((cc ^ (r & 7)) << 4);
      *reinterpret_cast<uint4*>(sP + off) = make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
      *reinterpret_cast<uint4*>(sdS + off) =
          make_uint4(dk2[4 * cc], dk2[4 * cc + 1], dk2[4 * cc + 2], dk2[4 * cc + 3]);
    }
    if (it + 1 < total) load_stats(it + 1);  // buffer (it+1)&1 was last read by chunk it-1's softmax
    fence_proxy_async_cta();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t qa = sQa + st * C::C_BYTES, da = sdOa + st * C::C_BYTES;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        umma_f16(tmem + C::DV_COL, sdesc_sw128(sPa + kk * 32, 16, 1024), sdesc_sw128(da + kk * 2048, 8192, 1024),
                 idesc_g, (it > 0 || kk > 0) ? 1u : 0u);
        umma_f16(tmem + C::DK_COL, sdesc_sw128(sdSa + kk * 32, 16, 1024), sdesc_sw128(qa + kk * 2048, 8192, 1024),
                 idesc_g, (it > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(gbar);
    }
  }

  if (ok && total > 0) {
    ok = mbar_wait(gbar, static_cast<uint32_t>((total - 1) & 1), abort_flag, err, kErrTimeoutFlag);
    ok = !__syncthreads_or(!ok);
  }
  if (ok && total > 0) {
    tc_fence_after();
    const bool row_ok = key < L;
    const int64_t orow = (static_cast<int64_t>(s0 + key) * Hkv + hk) * D;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const uint32_t col = which == 0 ? C::DV_COL : C::DK_COL;
      const float mul = which == 0 ? 1.f : scale;
      bf16* out = (which == 0 ? dV : dK) + orow;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 64) {
        uint32_t o[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld16(tmem + lane_base + col + c0 + 16 * c, o[c]);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              w[e] = pack_bf16x2(__uint_as_float(o[c][2 * e]) * mul, __uint_as_float(o[c][2 * e + 1]) * mul);
            uint4* dst = reinterpret_cast<uint4*>(out + c0 + 16 * c);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
      }
    }
  } else if (total == 0 && key < L) {
    // keys no query attends to (cannot happen for a non-empty segment; kept for completeness)
    const int64_t orow = (static_cast<int64_t>(s0 + key) * Hkv + hk) * D;
    for (int c = 0; c < D; ++c) dK[orow + c] = dV[orow + c] = f2bf(0.f);
  }
  if (!ok && tid == 0) {
    volatile int no_abort = 0;
    umma_commit(drain);
    mbar_wait(drain, 0, &no_abort, nullptr, 0);
    mbar_wait(kvbar, 0, &no_abort, nullptr, 0);
    for (int i = max(0, loads_issued - 2); i < loads_issued; ++i)
      mbar_wait(&qfull[i & 1], static_cast<uint32_t>((i >> 1) & 1), &no_abort, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, bool CAUSAL>
void launch_bwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                   const at::Tensor& lse, const at::Tensor& delta, const at::Tensor& cu, at::Tensor& dk, at::Tensor& dv,
                   int max_seqlen, float scale, const int* xq) {
  using C = TcBwdCfg<D>;
  const int B = static_cast<int>(cu.numel() - 1), Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(k.size(1));
  const int T = static_cast<int>(q.size(0));
  const CUtensorMap tq = make_tmap_2d_bf16(q.data_ptr(), static_cast<int64_t>(Hq) * D, T, static_cast<int64_t>(Hq) * D,
                                           64, 64);
  const CUtensorMap tdo = make_tmap_2d_bf16(dout.data_ptr(), static_cast<int64_t>(Hq) * D, T,
                                            static_cast<int64_t>(Hq) * D, 64, 64);
  const CUtensorMap tk = make_tmap_2d_bf16(k.data_ptr(), static_cast<int64_t>(Hkv) * D, T,
                                           static_cast<int64_t>(Hkv) * D, 64, kBM);
  const CUtensorMap tv = make_tmap_2d_bf16(v.data_ptr(), static_cast<int64_t>(Hkv) * D, T,
                                           static_cast<int64_t>(Hkv) * D, 64, kBM);
  auto kern = flash_bwd_dkdv_tc_kernel<D, CAUSAL>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  const dim3 grid((max_seqlen + kBM - 1) / kBM, Hkv, B);
  launch_pdl(kern, grid, dim3(128), C::SMEM, at::cuda::getCurrentCUDAStream(), tq, tk, tv, tdo, lse.data_ptr<float>(),
             delta.data_ptr<float>(), cu.data_ptr<int>(), reinterpret_cast<bf16*>(dk.data_ptr()),
             reinterpret_cast<bf16*>(dv.data_ptr()), Hq, Hkv, T, scale * kLog2eTc, scale, xq,
             err_word(q.device().index()));
}

}  // namespace

bool flash_attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
                       at::Tensor& o, at::Tensor& lse, int max_seqlen, bool causal, float scale, const int* pre) {
  static const bool enabled = [] {
    const char* e = std::getenv("VLMRL_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  const int D = static_cast<int>(q.size(2));
  if (!enabled || (D != 64 && D != 128)) return false;
  if (D == 128)
    causal ? launch_tc<128, true>(q, k, v, cu, o, lse, max_seqlen, scale, pre)
           : launch_tc<128, false>(q, k, v, cu, o, lse, max_seqlen, scale, pre);
  else
    causal ? launch_tc<64, true>(q, k, v, cu, o, lse, max_seqlen, scale, pre)
           : launch_tc<64, false>(q, k, v, cu, o, lse, max_seqlen, scale, pre);
  return true;
}

}  // namespace vlm

namespace vlm {

bool flash_attn_bwd_dkdv_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                            const at::Tensor& lse, const at::Tensor& delta, const at::Tensor& cu, at::Tensor& dk,
                            at::Tensor& dv, int max_seqlen, bool causal, float scale, const int* xq) {
  static const bool enabled = [] {
    const char* e = std::getenv("VLMRL_ATTN_BWD_TC");
    return e && e[0] == '1';
  }();
  const int D = static_cast<int>(q.size(2));
  if (!enabled || (D != 64 && D != 128)) return false;
  if (D == 128)
    causal ? launch_bwd_tc<128, true>(q, k, v, dout, lse, delta, cu, dk, dv, max_seqlen, scale, xq)
           : launch_bwd_tc<128, false>(q, k, v, dout, lse, delta, cu, dk, dv, max_seqlen, scale, xq);
  else
    causal ? launch_bwd_tc<64, true>(q, k, v, dout, lse, delta, cu, dk, dv, max_seqlen, scale, xq)
           : launch_bwd_tc<64, false>(q, k, v, dout, lse, delta, cu, dk, dv, max_seqlen, scale, xq);
  return true;
}

}  // namespace vlm
