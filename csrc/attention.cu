// Varlen GQA flash attention (forward + backward) and KV-cache decode attention.
//
// Forward: one CTA = 64 queries of one (sequence, q-head); 4 warps x 16 query rows;
// K/V tiles of 64 keys are double-buffered in swizzled shared memory with
// cp.async; S = Q.K^T and O += P.V run on bf16 mma.sync m16n8k16 with fp32
// accumulation; online softmax in base 2.  Outputs O (bf16) and the natural-log
// LSE [Hq, T] for the backward.
//
// Backward (no atomics): (1) delta = rowsum(dO * O); (2) one CTA per
// (sequence, 64-key block, kv-head) accumulates dK, dV over every q-head of the
// GQA group and every q block; (3) one CTA per (sequence, 64-query block, q-head)
// recomputes P and dP to form dQ.
//
// Decode: flash-decoding over the KV cache, one CTA per (kv-head, sequence,
// key split).  For head_dim 128 the K/V chunks arrive by 2-D TMA into swizzled
// tiles and both products run on mma.sync; other head sizes use 1-D bulk copies
// and warp-shuffle dot products.  A combine kernel merges key splits.
#include <ATen/cuda/CUDAContext.h>
#include <atomic>
#include <cstdlib>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "kv_layout.cuh"
#include "host_utils.h"
#include "mma_sync.cuh"
#include "vlm_noalloc.h"

namespace vlm {

using bf16 = __nv_bfloat16;

// [rows][D] bf16 tile with the 16-byte chunks of each row XOR-swizzled by the row index.
template <int D>
struct Tile {
  static constexpr int CH = D / 8;
  static constexpr int SW = CH < 8 ? CH : 8;
  VLM_DEV static int off(int row, int col) { return row * D + ((((col >> 3) ^ (row & (SW - 1)))) << 3) + (col & 7); }
};

// Load `rows` rows (row r from token t0+r of a [T, H, D] tensor at head h) into a swizzled tile; rows past `limit`
// are zero-filled.
template <int D>
VLM_DEV void load_rows(bf16* s, const bf16* g, int t0, int rows, int limit, int H, int h, int tid, int nthr) {
  constexpr int CH = D / 8;
  for (int i = tid; i < rows * CH; i += nthr) {
    const int r = i / CH, c = i % CH;
    const bool ok = t0 + r < limit;
    const bf16* src = g + ((static_cast<int64_t>(ok ? t0 + r : 0) * H + h) * D + c * 8);
    cp_async16(s + Tile<D>::off(r, c * 8), src, ok);
  }
}

// A fragment (16 x 16) at (r0, c0) of a swizzled [rows][D] tile.
template <int D>
VLM_DEV void frag_a(uint32_t (&a)[4], const bf16* s, int r0, int c0, int lane) {
  const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = c0 + (lane >> 4) * 8;
  ldsm_x4(a, s + Tile<D>::off(r, c));
}
// B fragments for two n-blocks (n0, n0+8) x k-step (k0..k0+15), where the tile is stored [n][k]
// (rows = n, contiguous k).  b[0],b[1] -> n-block n0; b[2],b[3] -> n-block n0+8.
template <int D>
VLM_DEV void frag_b_nk(uint32_t (&b)[4], const bf16* s, int n0, int k0, int lane) {
  const int r = n0 + (lane & 7) + (lane >> 4) * 8;
  const int c = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(b, s + Tile<D>::off(r, c));
}
// B fragments for two n-blocks (n0, n0+8) x k-step, where the tile is stored [k][n] (rows = k).
template <int D>
VLM_DEV void frag_b_kn(uint32_t (&b)[4], const bf16* s, int k0, int n0, int lane) {
  const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = n0 + (lane >> 4) * 8;
  ldsm_x4_t(b, s + Tile<D>::off(r, c));
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ------------------------------------------------------------------ forward
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_fwd_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                        const bf16* __restrict__ V, const int* __restrict__ cu,
                                                        bf16* __restrict__ O, float* __restrict__ LSE, int Hq, int Hkv,
                                                        int T, float scale_log2, const int* __restrict__ pre) {
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = cu[b], L = cu[b + 1] - s0;
  const int q0 = qb * 64;
  if (q0 >= L) return;
  // shared prefix: every query of this segment also sees keys [pstart, pstart + plen) (no causal mask)
  const int pstart = pre ? pre[2 * b] : 0, plen = pre ? pre[2 * b + 1] : 0;
  const int hk = h / (Hq / Hkv);
  extern __shared__ __align__(128) uint8_t smem_bytes[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_bytes);
  bf16* sK = sQ + 64 * D;
  bf16* sV = sK + 2 * 64 * D;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;

  const bf16* Qs = Q + static_cast<int64_t>(s0) * Hq * D;
  const bf16* Ks = K + static_cast<int64_t>(s0) * Hkv * D;
  const bf16* Vs = V + static_cast<int64_t>(s0) * Hkv * D;
  const bf16* Kp = K + static_cast<int64_t>(pstart) * Hkv * D;
  const bf16* Vp = V + static_cast<int64_t>(pstart) * Hkv * D;
  load_rows<D>(sQ, Qs, q0, 64, L, Hq, h, tid, 128);
  const int nkp = (plen + 63) / 64;
  const int nkb = nkp + (CAUSAL ? min((L + 63) / 64, qb + 1) : (L + 63) / 64);
  auto load_kv = [&](int j, int buf) {
    if (j < nkp) {
      load_rows<D>(sK + buf * 64 * D, Kp, j * 64, 64, plen, Hkv, hk, tid, 128);
      load_rows<D>(sV + buf * 64 * D, Vp, j * 64, 64, plen, Hkv, hk, tid, 128);
    } else {
      load_rows<D>(sK + buf * 64 * D, Ks, (j - nkp) * 64, 64, L, Hkv, hk, tid, 128);
      load_rows<D>(sV + buf * 64 * D, Vs, (j - nkp) * 64, 64, L, Hkv, hk, tid, 128);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_kv(j + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const bool in_pre = j < nkp;
    const int kbase = in_pre ? j * 64 : (j - nkp) * 64;
    const int klim = in_pre ? plen : L;
    const bf16* k_t = sK + buf * 64 * D;
    const bf16* v_t = sV + buf * 64 * D;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      frag_a<D>(a, sQ, warp * 16, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        frag_b_nk<D>(bb, k_t, np * 16, kk * 16, lane);
        mma_bf16(s[2 * np], a, bb[0], bb[1]);
        mma_bf16(s[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // scale + mask + online softmax
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kbase + nb * 8 + 2 * tq + e;
        const bool bad0 = key >= klim || (CAUSAL && !in_pre && key > row0);
        const bool bad1 = key >= klim || (CAUSAL && !in_pre && key > row1);
        s[nb][e] = bad0 ? -INFINITY : s[nb][e] * scale_log2;
        s[nb][2 + e] = bad1 ? -INFINITY : s[nb][2 + e] * scale_log2;
        mx0 = fmaxf(mx0, s[nb][e]);
        mx1 = fmaxf(mx1, s[nb][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      s[nb][0] = exp2f(s[nb][0] - base0);
      s[nb][1] = exp2f(s[nb][1] - base0);
      s[nb][2] = exp2f(s[nb][2] - base1);
      s[nb][3] = exp2f(s[nb][3] - base1);
      ps0 += s[nb][0] + s[nb][1];
      ps1 += s[nb][2] + s[nb][3];
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= al0;
      acc[i][1] *= al0;
      acc[i][2] *= al1;
      acc[i][3] *= al1;
    }
    // O += P . V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bb[4];
        frag_b_kn<D>(bb, v_t, kk * 16, dp * 16, lane);
        mma_bf16(acc[2 * dp], a, bb[0], bb[1]);
        mma_bf16(acc[2 * dp + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb) {
    const int col = nb * 8 + 2 * tq;
    if (row0 < L)
      *reinterpret_cast<uint32_t*>(O + ((static_cast<int64_t>(s0 + row0) * Hq + h) * D + col)) =
          pack_bf16x2(acc[nb][0] * inv0, acc[nb][1] * inv0);
    if (row1 < L)
      *reinterpret_cast<uint32_t*>(O + ((static_cast<int64_t>(s0 + row1) * Hq + h) * D + col)) =
          pack_bf16x2(acc[nb][2] * inv1, acc[nb][3] * inv1);
  }
  if (tq == 0) {
    if (row0 < L) LSE[static_cast<int64_t>(h) * T + s0 + row0] = l0 > 0.f ? (m0 + log2f(l0)) * kLn2 : -INFINITY;
    if (row1 < L) LSE[static_cast<int64_t>(h) * T + s0 + row1] = l1 > 0.f ? (m1 + log2f(l1)) * kLn2 : -INFINITY;
  }
}

// ------------------------------------------------------------------ backward: delta = rowsum(dO * O)
__global__ void attn_delta_kernel(const bf16* __restrict__ dO, const bf16* __restrict__ O, float* __restrict__ delta,
                                  int T, int H, int D) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(T) * H) return;
  const int t = static_cast<int>(w / H), h = static_cast<int>(w % H);
  const bf16* a = dO + w * D;
  const bf16* o = O + w * D;
  float s = 0.f;
  for (int c = lane; c < D; c += 32) s += bf2f(a[c]) * bf2f(o[c]);
  s = warp_sum(s);
  if (lane == 0) delta[static_cast<int64_t>(h) * T + t] = s;
}

// ------------------------------------------------------------------ backward: dK, dV
// CTA = (64-key block, kv-head, sequence); warp w owns keys [16w, 16w+16).  Queries are
// processed in chunks of 32 for every q-head of the GQA group.
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_bwd_dkdv_kernel(
    const bf16* __restrict__ Q, const bf16* __restrict__ K, const bf16* __restrict__ V, const bf16* __restrict__ dO,
    const float* __restrict__ LSE, const float* __restrict__ DELTA, const int* __restrict__ cu, bf16* __restrict__ dK,
    bf16* __restrict__ dV, int Hq, int Hkv, int T, float scale_log2, float scale, const int* __restrict__ xq) {
  constexpr int QC = 32;
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int s0 = cu[b], L = cu[b + 1] - s0;
  const int k0 = kb * 64;
  if (k0 >= L) return;
  // queries [xs, xs + xlen) outside this segment see all of its keys (segments sharing it as a prefix)
  const int xs = xq ? xq[2 * b] : 0, xlen = xq ? xq[2 * b + 1] - xq[2 * b] : 0;
  const int rep = Hq / Hkv;
  extern __shared__ __align__(128) uint8_t smem_bytes[];
  bf16* sK = reinterpret_cast<bf16*>(smem_bytes);
  bf16* sV = sK + 64 * D;
  bf16* sQ = sV + 64 * D;        // [2][QC][D]
  bf16* sdO = sQ + 2 * QC * D;   // [2][QC][D]
  float* sL = reinterpret_cast<float*>(sdO + 2 * QC * D);  // [2][QC]
  float* sDl = sL + 2 * QC;                                 // [2][QC]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const bf16* Ks = K + static_cast<int64_t>(s0) * Hkv * D;
  const bf16* Vs = V + static_cast<int64_t>(s0) * Hkv * D;
  const bf16* Qs = Q + static_cast<int64_t>(s0) * Hq * D;
  const bf16* dOs = dO + static_cast<int64_t>(s0) * Hq * D;
  load_rows<D>(sK, Ks, k0, 64, L, Hkv, hk, tid, 128);
  load_rows<D>(sV, Vs, k0, 64, L, Hkv, hk, tid, 128);
  cp_async_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int qc_start = CAUSAL ? k0 / QC : 0;
  const int qc_end = (L + QC - 1) / QC;
  const int n_own = qc_end - qc_start;
  const int n_chunks = n_own + (xlen + QC - 1) / QC;
  const int total = rep * n_chunks;
  const bf16* Qx = Q + static_cast<int64_t>(xs) * Hq * D;
  const bf16* dOx = dO + static_cast<int64_t>(xs) * Hq * D;
  auto issue = [&](int it, int buf) {
    const int hh = hk * rep + it / n_chunks;
    const int c = it % n_chunks;
    const bool own = c < n_own;
    const int qs = own ? (qc_start + c) * QC : (c - n_own) * QC;
    const int qlim = own ? L : xlen;
    const int abs0 = own ? s0 : xs;
    load_rows<D>(sQ + buf * QC * D, own ? Qs : Qx, qs, QC, qlim, Hq, hh, tid, 128);
    load_rows<D>(sdO + buf * QC * D, own ? dOs : dOx, qs, QC, qlim, Hq, hh, tid, 128);
    for (int i = tid; i < QC; i += 128) {
      const bool ok = qs + i < qlim;
      sL[buf * QC + i] = ok ? LSE[static_cast<int64_t>(hh) * T + abs0 + qs + i] * kLog2e : INFINITY;
      sDl[buf * QC + i] = ok ? DELTA[static_cast<int64_t>(hh) * T + abs0 + qs + i] : 0.f;
    }
  };
  if (total > 0) issue(0, 0);
  cp_async_commit();
  const int key_r0 = k0 + warp * 16 + g, key_r1 = key_r0 + 8;

  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    if (it + 1 < total) {
      __syncthreads();  // buffer buf^1 no longer read
      issue(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int c = it % n_chunks;
    const bool own = c < n_own;
    const int qs = own ? (qc_start + c) * QC : (c - n_own) * QC;
    const int qlim = own ? L : xlen;
    const bf16* q_t = sQ + buf * QC * D;
    const bf16* do_t = sdO + buf * QC * D;
    const float* lt = sL + buf * QC;
    const float* dlt = sDl + buf * QC;
    // S^T (16 keys x QC queries) = K_w . Q^T
    float st[QC / 8][4];
#pragma unroll
    for (int i = 0; i < QC / 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      frag_a<D>(a, sK, warp * 16, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < QC / 16; ++np) {
        uint32_t bb[4];
        frag_b_nk<D>(bb, q_t, np * 16, kk * 16, lane);
        mma_bf16(st[2 * np], a, bb[0], bb[1]);
        mma_bf16(st[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // P^T = exp2(S^T*scale - lse)
#pragma unroll
    for (int nb = 0; nb < QC / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int qi = nb * 8 + 2 * tq + e;
        const int qa = qs + qi;
        const bool bad0 = qa >= qlim || key_r0 >= L || (CAUSAL && own && qa < key_r0);
        const bool bad1 = qa >= qlim || key_r1 >= L || (CAUSAL && own && qa < key_r1);
        st[nb][e] = bad0 ? 0.f : exp2f(st[nb][e] * scale_log2 - lt[qi]);
        st[nb][2 + e] = bad1 ? 0.f : exp2f(st[nb][2 + e] * scale_log2 - lt[qi]);
      }
    }
    // dV += P^T . dO
#pragma unroll
    for (int kk = 0; kk < QC / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      a[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      a[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      a[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bb[4];
        frag_b_kn<D>(bb, do_t, kk * 16, dp * 16, lane);
        mma_bf16(dv[2 * dp], a, bb[0], bb[1]);
        mma_bf16(dv[2 * dp + 1], a, bb[2], bb[3]);
      }
    }
    // dP^T = V_w . dO^T
    float dpt[QC / 8][4];
#pragma unroll
    for (int i = 0; i < QC / 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      frag_a<D>(a, sV, warp * 16, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < QC / 16; ++np) {
        uint32_t bb[4];
        frag_b_nk<D>(bb, do_t, np * 16, kk * 16, lane);
        mma_bf16(dpt[2 * np], a, bb[0], bb[1]);
        mma_bf16(dpt[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // dS^T = P^T * (dP^T - delta)
#pragma unroll
    for (int nb = 0; nb < QC / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int qi = nb * 8 + 2 * tq + e;
        st[nb][e] = st[nb][e] * (dpt[nb][e] - dlt[qi]);
        st[nb][2 + e] = st[nb][2 + e] * (dpt[nb][2 + e] - dlt[qi]);
      }
    }
    // dK += dS^T . Q
#pragma unroll
    for (int kk = 0; kk < QC / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      a[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      a[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      a[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bb[4];
        frag_b_kn<D>(bb, q_t, kk * 16, dp * 16, lane);
        mma_bf16(dk[2 * dp], a, bb[0], bb[1]);
        mma_bf16(dk[2 * dp + 1], a, bb[2], bb[3]);
      }
    }
  }
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb) {
    const int col = nb * 8 + 2 * tq;
    if (key_r0 < L) {
      const int64_t o = (static_cast<int64_t>(s0 + key_r0) * Hkv + hk) * D + col;
      *reinterpret_cast<uint32_t*>(dK + o) = pack_bf16x2(dk[nb][0] * scale, dk[nb][1] * scale);
      *reinterpret_cast<uint32_t*>(dV + o) = pack_bf16x2(dv[nb][0], dv[nb][1]);
    }
    if (key_r1 < L) {
      const int64_t o = (static_cast<int64_t>(s0 + key_r1) * Hkv + hk) * D + col;
      *reinterpret_cast<uint32_t*>(dK + o) = pack_bf16x2(dk[nb][2] * scale, dk[nb][3] * scale);
      *reinterpret_cast<uint32_t*>(dV + o) = pack_bf16x2(dv[nb][2], dv[nb][3]);
    }
  }
}

// ------------------------------------------------------------------ backward: dQ
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_bwd_dq_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                           const bf16* __restrict__ V, const bf16* __restrict__ dO,
                                                           const float* __restrict__ LSE,
                                                           const float* __restrict__ DELTA, const int* __restrict__ cu,
                                                           bf16* __restrict__ dQ, int Hq, int Hkv, int T,
                                                           float scale_log2, float scale, const int* __restrict__ pre) {
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = cu[b], L = cu[b + 1] - s0;
  const int q0 = qb * 64;
  if (q0 >= L) return;
  const int pstart = pre ? pre[2 * b] : 0, plen = pre ? pre[2 * b + 1] : 0;
  const int hk = h / (Hq / Hkv);
  extern __shared__ __align__(128) uint8_t smem_bytes[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_bytes);
  bf16* sdO = sQ + 64 * D;
  bf16* sK = sdO + 64 * D;  // [2][64][D]
  bf16* sV = sK + 2 * 64 * D;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const bf16* Ks = K + static_cast<int64_t>(s0) * Hkv * D;
  const bf16* Vs = V + static_cast<int64_t>(s0) * Hkv * D;
  load_rows<D>(sQ, Q + static_cast<int64_t>(s0) * Hq * D, q0, 64, L, Hq, h, tid, 128);
  load_rows<D>(sdO, dO + static_cast<int64_t>(s0) * Hq * D, q0, 64, L, Hq, h, tid, 128);
  const bf16* Kp = K + static_cast<int64_t>(pstart) * Hkv * D;
  const bf16* Vp = V + static_cast<int64_t>(pstart) * Hkv * D;
  const int nkp = (plen + 63) / 64;
  auto load_kv = [&](int j, int buf) {
    if (j < nkp) {
      load_rows<D>(sK + buf * 64 * D, Kp, j * 64, 64, plen, Hkv, hk, tid, 128);
      load_rows<D>(sV + buf * 64 * D, Vp, j * 64, 64, plen, Hkv, hk, tid, 128);
    } else {
      load_rows<D>(sK + buf * 64 * D, Ks, (j - nkp) * 64, 64, L, Hkv, hk, tid, 128);
      load_rows<D>(sV + buf * 64 * D, Vs, (j - nkp) * 64, 64, L, Hkv, hk, tid, 128);
    }
  };
  load_kv(0, 0);
  cp_async_commit();
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  const float lse0 = row0 < L ? LSE[static_cast<int64_t>(h) * T + s0 + row0] * kLog2e : INFINITY;
  const float lse1 = row1 < L ? LSE[static_cast<int64_t>(h) * T + s0 + row1] * kLog2e : INFINITY;
  const float dl0 = row0 < L ? DELTA[static_cast<int64_t>(h) * T + s0 + row0] : 0.f;
  const float dl1 = row1 < L ? DELTA[static_cast<int64_t>(h) * T + s0 + row1] : 0.f;
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const int nkb = nkp + (CAUSAL ? min((L + 63) / 64, qb + 1) : (L + 63) / 64);
  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_kv(j + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const bool in_pre = j < nkp;
    const int kbase = in_pre ? j * 64 : (j - nkp) * 64;
    const int klim = in_pre ? plen : L;
    const bf16* k_t = sK + buf * 64 * D;
    const bf16* v_t = sV + buf * 64 * D;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], ad[4];
      frag_a<D>(a, sQ, warp * 16, kk * 16, lane);
      frag_a<D>(ad, sdO, warp * 16, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4], bv[4];
        frag_b_nk<D>(bb, k_t, np * 16, kk * 16, lane);
        frag_b_nk<D>(bv, v_t, np * 16, kk * 16, lane);
        mma_bf16(s[2 * np], a, bb[0], bb[1]);
        mma_bf16(s[2 * np + 1], a, bb[2], bb[3]);
        mma_bf16(dp[2 * np], ad, bv[0], bv[1]);
        mma_bf16(dp[2 * np + 1], ad, bv[2], bv[3]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kbase + nb * 8 + 2 * tq + e;
        const bool bad0 = key >= klim || row0 >= L || (CAUSAL && !in_pre && key > row0);
        const bool bad1 = key >= klim || row1 >= L || (CAUSAL && !in_pre && key > row1);
        const float p0 = bad0 ? 0.f : exp2f(s[nb][e] * scale_log2 - lse0);
        const float p1 = bad1 ? 0.f : exp2f(s[nb][2 + e] * scale_log2 - lse1);
        s[nb][e] = p0 * (dp[nb][e] - dl0);
        s[nb][2 + e] = p1 * (dp[nb][2 + e] - dl1);
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dd = 0; dd < D / 16; ++dd) {
        uint32_t bb[4];
        frag_b_kn<D>(bb, k_t, kk * 16, dd * 16, lane);
        mma_bf16(dq[2 * dd], a, bb[0], bb[1]);
        mma_bf16(dq[2 * dd + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb) {
    const int col = nb * 8 + 2 * tq;
    if (row0 < L)
      *reinterpret_cast<uint32_t*>(dQ + ((static_cast<int64_t>(s0 + row0) * Hq + h) * D + col)) =
          pack_bf16x2(dq[nb][0] * scale, dq[nb][1] * scale);
    if (row1 < L)
      *reinterpret_cast<uint32_t*>(dQ + ((static_cast<int64_t>(s0 + row1) * Hq + h) * D + col)) =
          pack_bf16x2(dq[nb][2] * scale, dq[nb][3] * scale);
  }
}

// ------------------------------------------------------------------ decode attention (flash-decoding)
// q [B, Hq, D], caches [B, Hkv, Tmax, D], len [B] -> o [B, Hq, D].
// CTA = (kv-head, sequence, key split), NW warps.  The keys of a (sequence, kv-head) are contiguous rows of
// the cache, so thread 0 streams them with 1-D TMA bulk copies (KC keys of K and of V per stage) into a
// STAGES-deep shared-memory ring whose mbarriers the warps wait on (bounded).  Warp w scores keys
// w, w+NW, ... of each stage for the REP q-heads of the group (lane l owns D/32 dims, warp-shuffle
// reduction) and keeps its own online softmax; warps merge in shared memory at the end.  With more than
// one split the CTA writes (max, sum, unnormalised acc) and decode_combine_kernel finishes.
template <int D, int REP, int NW = 8, int KC = 32, int STAGES = 4>
__global__ void __launch_bounds__(NW * 32) decode_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                              const bf16* __restrict__ vc, const int* __restrict__ lens,
                                                              bf16* __restrict__ o, float* __restrict__ part, int Hq,
                                                              KvLayout lay, float scale_log2, int splits,
                                                              int* err) {
  static_assert(kKvBlock % KC == 0, "a key chunk must not straddle a cache block");
  constexpr int ND = D / 32;
  constexpr int KPW = KC / NW;  // keys per warp per stage
  constexpr int CHUNK = KC * D * 2;
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  bf16* sK = reinterpret_cast<bf16*>(dsm_raw);
  bf16* sV = sK + STAGES * KC * D;
  uint64_t* full = reinterpret_cast<uint64_t*>(sV + STAGES * KC * D);
  float* sm_m = reinterpret_cast<float*>(full + STAGES);    // [NW][REP]
  float* sm_l = sm_m + NW * REP;                             // [NW][REP]
  float* sm_acc = sm_l + NW * REP;                           // [NW][REP][D]
  __shared__ int abort_flag;

  pdl_wait();
  pdl_trigger();
  const int hk = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  const int L = min(lens[b], lay.cap);
  int per = (L + splits - 1) / splits;
  if (lay.table) per = (per + kKvBlock - 1) / kKvBlock * kKvBlock;  // splits start on block boundaries
  const int k0 = sp * per, k1 = min(L, k0 + per);
  const int nk = max(0, k1 - k0);
  const int nchunks = (nk + KC - 1) / KC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int st = c % STAGES;
    const int keys = min(KC, nk - c * KC);
    const uint32_t bytes = static_cast<uint32_t>(keys) * D * 2;
    // the chunk's keys are consecutive rows of one (sequence or block, head) run
    const int64_t row = kv_row(lay, b, hk, k0 + c * KC);
    mbar_arrive_expect_tx(&full[st], 2 * bytes);
    bulk_load(sK + st * KC * D, kc + row * D, bytes, &full[st]);
    bulk_load(sV + st * KC * D, vc + row * D, bytes, &full[st]);
  };
  if (threadIdx.x == 0)
    for (int c = 0; c < STAGES && c < nchunks; ++c) issue(c);

  float qv[REP][ND];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const bf16* qr = q + (static_cast<int64_t>(b) * Hq + hk * REP + r) * D + lane * ND;
#pragma unroll
    for (int j = 0; j < ND; ++j) qv[r][j] = bf2f(qr[j]) * scale_log2;
  }
  float m[REP], l[REP], acc[REP][ND];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int j = 0; j < ND; ++j) acc[r][j] = 0.f;
  }
  auto load_nd = [&](const bf16* src, float (&out)[ND]) {
    if constexpr (ND == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(src);
      const float2 a = unpack_bf16x2(u.x), c = unpack_bf16x2(u.y);
      out[0] = a.x; out[1] = a.y; out[2] = c.x; out[3] = c.y;
    } else if constexpr (ND == 2) {
      const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src));
      out[0] = a.x; out[1] = a.y;
    } else {
#pragma unroll
      for (int j = 0; j < ND; ++j) out[j] = bf2f(src[j]);
    }
  };
  int consumed = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % STAGES;
    if (!mbar_wait(&full[st], static_cast<uint32_t>((c / STAGES) & 1), &abort_flag, err, kErrTimeoutFlag)) break;
    consumed = c + 1;
    const int keys = min(KC, nk - c * KC);
    const bf16* ks = sK + st * KC * D + lane * ND;
    const bf16* vs = sV + st * KC * D + lane * ND;
    float kv[KPW][ND], vv[KPW][ND];
    bool ok[KPW];
#pragma unroll
    for (int u = 0; u < KPW; ++u) {
      const int t = warp + u * NW;
      ok[u] = t < keys;
      if (ok[u]) {
        load_nd(ks + t * D, kv[u]);
        load_nd(vs + t * D, vv[u]);
      } else {
#pragma unroll
        for (int j = 0; j < ND; ++j) kv[u][j] = vv[u][j] = 0.f;
      }
    }
    float sc[KPW][REP];
#pragma unroll
    for (int u = 0; u < KPW; ++u)
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float x = 0.f;
#pragma unroll
        for (int j = 0; j < ND; ++j) x += qv[r][j] * kv[u][j];
        sc[u][r] = x;
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < KPW; ++u)
#pragma unroll
        for (int r = 0; r < REP; ++r) sc[u][r] += __shfl_xor_sync(0xffffffffu, sc[u][r], off);
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float mx = m[r];
#pragma unroll
      for (int u = 0; u < KPW; ++u)
        if (ok[u]) mx = fmaxf(mx, sc[u][r]);
      const float cf = mx == -INFINITY ? 1.f : exp2f(m[r] - mx);
      l[r] *= cf;
#pragma unroll
      for (int j = 0; j < ND; ++j) acc[r][j] *= cf;
#pragma unroll
      for (int u = 0; u < KPW; ++u) {
        const float pr = ok[u] ? exp2f(sc[u][r] - mx) : 0.f;
        l[r] += pr;
#pragma unroll
        for (int j = 0; j < ND; ++j) acc[r][j] += pr * vv[u][j];
      }
      m[r] = mx;
    }
    __syncthreads();  // stage st fully consumed
    if (threadIdx.x == 0 && c + STAGES < nchunks) issue(c + STAGES);
  }
  if (abort_flag) {
    // drain this CTA's in-flight bulk copies before it exits
    if (threadIdx.x == 0) {
      const int issued = min(nchunks, consumed + STAGES);
      for (int c = consumed; c < issued; ++c) {
        volatile int no_abort = 0;
        mbar_wait(&full[c % STAGES], static_cast<uint32_t>((c / STAGES) & 1), &no_abort, nullptr, 0);
      }
    }
    return;
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      sm_m[warp * REP + r] = m[r];
      sm_l[warp * REP + r] = l[r];
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int j = 0; j < ND; ++j) sm_acc[(warp * REP + r) * D + lane * ND + j] = acc[r][j];
  __syncthreads();
  for (int i = threadIdx.x; i < REP * D; i += NW * 32) {
    const int r = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, sm_m[w * REP + r]);
    float lt = 0.f, at = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float cf = sm_m[w * REP + r] == -INFINITY ? 0.f : exp2f(sm_m[w * REP + r] - mx);
      lt += sm_l[w * REP + r] * cf;
      at += sm_acc[(w * REP + r) * D + d] * cf;
    }
    const int h = hk * REP + r;
    if (splits == 1) {
      o[(static_cast<int64_t>(b) * Hq + h) * D + d] = f2bf(lt > 0.f ? at / lt : 0.f);
    } else {
      float* pp = part + ((static_cast<int64_t>(b) * Hq + h) * splits + sp) * (D + 2);
      pp[2 + d] = at;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = lt;
      }
    }
  }
}

// Tensor-core decode attention (head_dim 128).  CTA = (kv-head, sequence, key split), 4 warps.
// K and V chunks of 64 keys arrive by 2-D TMA as two 64x64 bf16 boxes each (128-byte swizzle, the same
// XOR layout as Tile<64>), STAGES deep.  Warp w owns keys [16w, 16w+16) of every chunk:
// S = Q.K^T with the REP query heads of the group as rows 0..REP-1 of a 16-row mma.sync tile,
// online softmax per head row, O += P.V; the four warps merge through shared memory at the end.
template <int REP, int STAGES = 3>
__global__ void __launch_bounds__(128) decode_attn_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                                                             const __grid_constant__ CUtensorMap tmV,
                                                             const bf16* __restrict__ q, const int* __restrict__ lens,
                                                             bf16* __restrict__ o, float* __restrict__ part, int Hq,
                                                             KvLayout lay, float scale_log2, int splits, int* err,
                                                             L2Prefetch pf, const int* __restrict__ lead,
                                                             const int* __restrict__ share_len) {
  constexpr int D = 128, KC = 64;
  static_assert(KC == kKvBlock, "one TMA box of keys per cache block");
  constexpr int HALF = KC * 64;  // elements of one 64x64 box
  extern __shared__ __align__(1024) uint8_t tc_raw[];
  bf16* sm = reinterpret_cast<bf16*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  bf16* sK = sm;                       // [STAGES][2 halves][64][64]
  bf16* sV = sK + STAGES * 2 * HALF;
  uint64_t* full = reinterpret_cast<uint64_t*>(sV + STAGES * 2 * HALF);
  float* red = reinterpret_cast<float*>(full + STAGES);  // merge area [4][REP][D + 2]
  __shared__ int abort_flag;
  l2_prefetch_share(pf);
  // Read before the grid dependency resolves: the lengths, the block table and the row-sharing fields are
  // written before the previous kernel starts (a decode step writes them before its first layer).
  const int hk = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  const int L = min(lens[b], lay.cap);
  int per = (L + splits - 1) / splits;
  if (lay.table) per = (per + kKvBlock - 1) / kKvBlock * kKvBlock;  // splits start on block boundaries
  const int k0 = sp * per, k1 = min(L, k0 + per);
  const int nk = max(0, k1 - k0);
  const int nchunks = (nk + KC - 1) / KC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  // Shared prompt (GRPO groups): keys [0, share_len[b]) of row b equal those of row lead[b], so whole
  // chunks inside that range are read from the leader's row; the group's CTAs then hit the same lines in
  // L2 instead of streaming identical copies from HBM.
  const int src_lead = lead ? lead[b] : b;
  const int src_share = share_len ? share_len[b] : 0;
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int st = c % STAGES;
    mbar_arrive_expect_tx(&full[st], 4 * HALF * 2);
    const int t0 = k0 + c * KC;
    const int y = static_cast<int>(kv_row(lay, t0 + KC <= src_share ? src_lead : b, hk, t0));
    tma_load_2d(sK + (st * 2 + 0) * HALF, &tmK, &full[st], 0, y);
    tma_load_2d(sK + (st * 2 + 1) * HALF, &tmK, &full[st], 64, y);
    tma_load_2d(sV + (st * 2 + 0) * HALF, &tmV, &full[st], 0, y);
    tma_load_2d(sV + (st * 2 + 1) * HALF, &tmV, &full[st], 64, y);
  };
  // Chunks wholly below the newest key (index L - 1) are issued before the grid dependency resolves: the
  // kernel before this one (dec_qkv in a decode step) appends only that key, so the cached prefix can
  // stream while it runs.  A predecessor that writes other keys must not trigger its dependents early.
  int early = 0;
  while (early < STAGES && early < nchunks && k0 + (early + 1) * KC <= L - 1) ++early;
  if (tid == 0)
    for (int c = 0; c < early; ++c) issue(c);
  pdl_wait();
  pdl_trigger();
  if (tid == 0)
    for (int c = early; c < STAGES && c < nchunks; ++c) issue(c);
  // Q fragments: rows g < REP are the group's heads, the rest zero
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    qa[kk][1] = qa[kk][3] = 0u;
    if (g < REP) {
      const bf16* qr = q + (static_cast<int64_t>(b) * Hq + hk * REP + g) * D + kk * 16 + 2 * tq;
      qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr) ;
      qa[kk][2] = *reinterpret_cast<const uint32_t*>(qr + 8);
    } else {
      qa[kk][0] = qa[kk][2] = 0u;
    }
  }
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m = -INFINITY, l = 0.f;  // running stats of row g (only rows g < REP are real)
  int consumed = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % STAGES;
    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>((c / STAGES) & 1), &abort_flag, err, kErrTimeoutFlag);
    if (__syncthreads_or(!ok)) break;  // every thread leaves at the same chunk
    consumed = c + 1;
    const bf16* kt = sK + st * 2 * HALF;
    bf16* vt = sV + st * 2 * HALF;
    if ((c + 1) * KC > nk) {
      // keys past this split's range: their V rows may hold anything (other sequences, unwritten
      // cache slots), and P = 0 does not cancel a NaN there, so zero them; only the last chunk is
      // partial and no later copy targets its stage.
      for (int i = lane; i < 16 * 16; i += 32) {
        const int r = warp * 16 + (i >> 4), ch = i & 15;
        if (c * KC + r >= nk) reinterpret_cast<uint4*>(vt + (ch >> 3) * HALF + r * 64)[ch & 7] = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    float s[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t bb[4];
      frag_b_nk<64>(bb, kt + (kk >> 2) * HALF, warp * 16, (kk & 3) * 16, lane);
      mma_bf16(s[0], qa[kk], bb[0], bb[1]);
      mma_bf16(s[1], qa[kk], bb[2], bb[3]);
    }
    const int kbase = c * KC + warp * 16;
    float mx = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = kbase + nb * 8 + 2 * tq + e < nk;
        s[nb][e] = ok ? s[nb][e] * scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[nb][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float base = mn == -INFINITY ? 0.f : mn;
    const float cf = exp2f(m - base);
    float ps = 0.f;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[nb][e] = exp2f(s[nb][e] - base);
        ps += s[nb][e];
      }
    l = l * cf + ps;
    m = mn;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= cf;
      acc[i][1] *= cf;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[0][0], s[0][1]);
    pa[1] = 0u;
    pa[2] = pack_bf16x2(s[1][0], s[1][1]);
    pa[3] = 0u;
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t bb[4];
      frag_b_kn<64>(bb, vt + (dp >> 2) * HALF, warp * 16, (dp & 3) * 16, lane);
      mma_bf16(acc[2 * dp], pa, bb[0], bb[1]);
      mma_bf16(acc[2 * dp + 1], pa, bb[2], bb[3]);
    }
    __syncthreads();
    if (tid == 0 && c + STAGES < nchunks) issue(c + STAGES);
  }
  if (consumed < nchunks) {  // aborted: drain the copies still in flight, then leave
    if (tid == 0) {
      const int issued = min(nchunks, consumed + STAGES);
      for (int c = consumed; c < issued; ++c) {
        volatile int no_abort = 0;
        mbar_wait(&full[c % STAGES], static_cast<uint32_t>((c / STAGES) & 1), &no_abort, nullptr, 0);
      }
    }
    return;
  }
  // per-warp row sums, then merge the four warps
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  float* rw = red + warp * REP * (D + 2);
  if (g < REP) {
    if (tq == 0) {
      rw[g * (D + 2)] = m;
      rw[g * (D + 2) + 1] = l;
    }
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      rw[g * (D + 2) + 2 + nb * 8 + 2 * tq] = acc[nb][0];
      rw[g * (D + 2) + 2 + nb * 8 + 2 * tq + 1] = acc[nb][1];
    }
  }
  __syncthreads();
  for (int i = tid; i < REP * D; i += 128) {
    const int r = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, red[(w * REP + r) * (D + 2)]);
    float lt = 0.f, at = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* e = red + (w * REP + r) * (D + 2);
      const float cfw = e[0] == -INFINITY ? 0.f : exp2f(e[0] - mx);
      lt += e[1] * cfw;
      at += e[2 + d] * cfw;
    }
    const int h = hk * REP + r;
    if (splits == 1) {
      o[(static_cast<int64_t>(b) * Hq + h) * D + d] = f2bf(lt > 0.f ? at / lt : 0.f);
    } else {
      float* pp = part + ((static_cast<int64_t>(b) * Hq + h) * splits + sp) * (D + 2);
      pp[2 + d] = at;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = lt;
      }
    }
  }
}

// Merges the key splits of decode_attn_kernel: part [B, Hq, splits, 2 + D] -> o [B, Hq, D].
__global__ void decode_combine_kernel(const float* __restrict__ part, bf16* __restrict__ o, int BH, int splits, int D) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x;
  if (bh >= BH) return;
  const float* p = part + static_cast<int64_t>(bh) * splits * (D + 2);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, p[s * (D + 2)]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float lt = 0.f, at = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = p[s * (D + 2)];
      const float c = ms == -INFINITY ? 0.f : exp2f(ms - mx);
      lt += p[s * (D + 2) + 1] * c;
      at += p[s * (D + 2) + 2 + d] * c;
    }
    o[static_cast<int64_t>(bh) * D + d] = f2bf(lt > 0.f ? at / lt : 0.f);
  }
}

// ------------------------------------------------------------------ host
template <typename KernT>
static void set_smem(KernT k, int bytes) {
  VLM_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <int D>
static void fwd_dispatch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
                         at::Tensor& o, at::Tensor& lse, int max_seqlen, bool causal, float scale, const int* pre) {
  const int B = static_cast<int>(cu.numel() - 1), Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(k.size(1));
  const int T = static_cast<int>(q.size(0));
  const dim3 grid((max_seqlen + 63) / 64, Hq, B);
  const int smem = 5 * 64 * D * 2;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto args = std::make_tuple(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
                              reinterpret_cast<const bf16*>(v.data_ptr()), cu.data_ptr<int>(),
                              reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), Hq, Hkv, T,
                              scale * kLog2e, pre);
  if (causal) {
    auto kern = flash_fwd_kernel<D, true>;
    set_smem(kern, smem);
    std::apply([&](auto... a) { kern<<<grid, 128, smem, st>>>(a...); }, args);
  } else {
    auto kern = flash_fwd_kernel<D, false>;
    set_smem(kern, smem);
    std::apply([&](auto... a) { kern<<<grid, 128, smem, st>>>(a...); }, args);
  }
  VLM_LAUNCHED();
}

static const int* seg_ptr(const c10::optional<at::Tensor>& t, const at::Tensor& cu, const char* what) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous() && t->numel() == 2 * (cu.numel() - 1) &&
                  t->device() == cu.device(),
              "attn: ", what, " must be int32 [segments, 2] on the device of cu_seqlens");
  return t->data_ptr<int>();
}

// attention_tc.cu: the tcgen05 forward for head_dim 64 / 128 (false: not handled, use the kernels here)
bool flash_attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
                       at::Tensor& o, at::Tensor& lse, int max_seqlen, bool causal, float scale, const int* pre);
// attention_tc.cu: dK / dV on tcgen05 for head_dim 64 / 128 (false: not handled)
bool flash_attn_bwd_dkdv_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                            const at::Tensor& lse, const at::Tensor& delta, const at::Tensor& cu, at::Tensor& dk,
                            at::Tensor& dv, int max_seqlen, bool causal, float scale, const int* xq);

// pre[b] = (start, len): keys every query of segment b also attends to (a shared prefix).
void flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu, at::Tensor o, at::Tensor lse,
                    int64_t max_seqlen, bool causal, double scale, c10::optional<at::Tensor> pre) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && o.is_contiguous(), "attn: contiguous");
  TORCH_CHECK(cu.scalar_type() == at::kInt, "attn: cu_seqlens int32");
  TORCH_CHECK(q.size(1) % k.size(1) == 0, "attn: Hq must be a multiple of Hkv");
  if (q.size(0) == 0 || max_seqlen == 0) return;
  const c10::cuda::CUDAGuard g(q.device());
  const int D = static_cast<int>(q.size(2));
  const int* pp = seg_ptr(pre, cu, "pre");
  const int ms = static_cast<int>(max_seqlen);
  const float sc = static_cast<float>(scale);
  if (flash_attn_fwd_tc(q, k, v, cu, o, lse, ms, causal, sc, pp)) return;
  switch (D) {
    case 16: fwd_dispatch<16>(q, k, v, cu, o, lse, ms, causal, sc, pp); break;
    case 32: fwd_dispatch<32>(q, k, v, cu, o, lse, ms, causal, sc, pp); break;
    case 64: fwd_dispatch<64>(q, k, v, cu, o, lse, ms, causal, sc, pp); break;
    case 128: fwd_dispatch<128>(q, k, v, cu, o, lse, ms, causal, sc, pp); break;
    default: TORCH_CHECK(false, "attn: unsupported head_dim ", D);
  }
}

template <int D>
static void bwd_dispatch(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const at::Tensor& lse, const at::Tensor& delta, const at::Tensor& cu, at::Tensor& dq,
                         at::Tensor& dk, at::Tensor& dv, int max_seqlen, bool causal, float scale, const int* pre,
                         const int* xq) {
  const int B = static_cast<int>(cu.numel() - 1), Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(k.size(1));
  const int T = static_cast<int>(q.size(0));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float sl2 = scale * kLog2e;
  if (!flash_attn_bwd_dkdv_tc(q, k, v, dout, lse, delta, cu, dk, dv, max_seqlen, causal, scale, xq)) {
    const dim3 grid((max_seqlen + 63) / 64, Hkv, B);
    const int smem = (2 * 64 * D + 4 * 32 * D) * 2 + 4 * 32 * 4;
    auto kern = causal ? flash_bwd_dkdv_kernel<D, true> : flash_bwd_dkdv_kernel<D, false>;
    set_smem(kern, smem);
    kern<<<grid, 128, smem, st>>>(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
                                  reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
                                  lse.data_ptr<float>(), delta.data_ptr<float>(), cu.data_ptr<int>(),
                                  reinterpret_cast<bf16*>(dk.data_ptr()), reinterpret_cast<bf16*>(dv.data_ptr()), Hq, Hkv, T,
                                  sl2, scale, xq);
    VLM_LAUNCHED();
  }
  {
    const dim3 grid((max_seqlen + 63) / 64, Hq, B);
    const int smem = 6 * 64 * D * 2;
    auto kern = causal ? flash_bwd_dq_kernel<D, true> : flash_bwd_dq_kernel<D, false>;
    set_smem(kern, smem);
    kern<<<grid, 128, smem, st>>>(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
                                  reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
                                  lse.data_ptr<float>(), delta.data_ptr<float>(), cu.data_ptr<int>(),
                                  reinterpret_cast<bf16*>(dq.data_ptr()), Hq, Hkv, T, sl2, scale, pre);
    VLM_LAUNCHED();
  }
}

// xq[b] = (start, end): queries outside segment b that attend to all of its keys (the inverse of pre).
void flash_attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                    at::Tensor cu, at::Tensor dq, at::Tensor dk, at::Tensor dv, int64_t max_seqlen, bool causal,
                    double scale, c10::optional<at::Tensor> pre, c10::optional<at::Tensor> xq) {
  TORCH_CHECK(dout.is_contiguous() && q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && o.is_contiguous(),
              "attn bwd: contiguous");
  if (q.size(0) == 0 || max_seqlen == 0) return;
  const c10::cuda::CUDAGuard g(q.device());
  const int T = static_cast<int>(q.size(0)), Hq = static_cast<int>(q.size(1)), D = static_cast<int>(q.size(2));
  at::Tensor delta = at::empty({Hq, T}, q.options().dtype(at::kFloat));
  const int64_t warps = static_cast<int64_t>(T) * Hq;
  attn_delta_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(dout.data_ptr()), reinterpret_cast<const bf16*>(o.data_ptr()), delta.data_ptr<float>(),
      T, Hq, D);
  VLM_LAUNCHED();
  const int ms = static_cast<int>(max_seqlen);
  const float sc = static_cast<float>(scale);
  const int* pp = seg_ptr(pre, cu, "pre");
  const int* xp = seg_ptr(xq, cu, "xq");
  TORCH_CHECK((pp == nullptr) == (xp == nullptr), "attn bwd: pass both pre and xq, or neither");
  switch (D) {
    case 16: bwd_dispatch<16>(dout, q, k, v, lse, delta, cu, dq, dk, dv, ms, causal, sc, pp, xp); break;
    case 32: bwd_dispatch<32>(dout, q, k, v, lse, delta, cu, dq, dk, dv, ms, causal, sc, pp, xp); break;
    case 64: bwd_dispatch<64>(dout, q, k, v, lse, delta, cu, dq, dk, dv, ms, causal, sc, pp, xp); break;
    case 128: bwd_dispatch<128>(dout, q, k, v, lse, delta, cu, dq, dk, dv, ms, causal, sc, pp, xp); break;
    default: TORCH_CHECK(false, "attn bwd: unsupported head_dim ", D);
  }
}

template <int D, int REP>
static void decode_dispatch(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& lens,
                            at::Tensor& o, float scale, const KvLayout& lay) {
  constexpr int NW = 8, KC = 32, STAGES = 4;
  const int B = static_cast<int>(q.size(0)), Hq = static_cast<int>(q.size(1)), Hkv = lay.Hkv;
  const int Tmax = lay.cap;
  const int sms = num_sms(q.device().index());
  // ~3 CTAs per SM; each split keeps >= 2 chunks of keys
  const int splits = std::max(1, std::min((3 * sms + B * Hkv - 1) / (B * Hkv), Tmax / (2 * KC)));
  const int smem = 2 * STAGES * KC * D * 2 + STAGES * 8 + (2 * NW * REP + NW * REP * D) * 4;
  auto kern = decode_attn_kernel<D, REP, NW, KC, STAGES>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  at::Tensor part;
  if (splits > 1) part = at::empty({B, Hq, splits, D + 2}, q.options().dtype(at::kFloat));
  launch_pdl(kern, dim3(Hkv, B, splits), dim3(NW * 32), smem, st, reinterpret_cast<const bf16*>(q.data_ptr()),
             reinterpret_cast<const bf16*>(kc.data_ptr()), reinterpret_cast<const bf16*>(vc.data_ptr()),
             lens.data_ptr<int>(), reinterpret_cast<bf16*>(o.data_ptr()), splits > 1 ? part.data_ptr<float>() : nullptr,
             Hq, lay, scale * kLog2e, splits, err_word(q.device().index()));
  if (splits > 1) {
    launch_pdl(decode_combine_kernel, dim3(B * Hq), dim3(128), 0, st, part.data_ptr<float>(),
               reinterpret_cast<bf16*>(o.data_ptr()), B * Hq, splits, D);
  }
}

template <int REP>
static void decode_tc_dispatch(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& lens,
                               at::Tensor& o, float scale, L2Prefetch pf, const int* lead, const int* share_len,
                               const KvLayout& lay) {
  constexpr int STAGES = 3, D = 128;
  const int B = static_cast<int>(q.size(0)), Hq = static_cast<int>(q.size(1)), Hkv = lay.Hkv;
  const int Tmax = lay.cap;
  const int sms = num_sms(q.device().index());
  // Key splits: enough CTAs for two per SM.  (Forcing two splits whenever one split leaves a partial last
  // wave measured slower: 4.70 vs 4.36 ms per 4B decode step at batch 64, cache length 390.)
  // VLMRL_DECODE_SPLITS overrides the count (measurements only).
  int splits = std::max(1, std::min((2 * sms + B * Hkv - 1) / (B * Hkv), Tmax / 128));
  if (const char* e = std::getenv("VLMRL_DECODE_SPLITS")) splits = std::max(1, std::atoi(e));
  const int smem = 1024 + STAGES * 4 * 64 * 64 * 2 + STAGES * 8 + 4 * REP * (D + 2) * 4;
  const int64_t rows = kc.size(0) * kc.size(1) * kc.size(2);  // every row of the layer (or of the block pool)
  TORCH_CHECK(rows < (int64_t(1) << 31), "decode_attn: cache layer too large for 32-bit TMA rows");
  const CUtensorMap tk = make_tmap_2d_bf16(kc.data_ptr(), D, rows, D, 64, 64);
  const CUtensorMap tv = make_tmap_2d_bf16(vc.data_ptr(), D, rows, D, 64, 64);
  auto kern = decode_attn_tc_kernel<REP, STAGES>;
  VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  at::Tensor part;
  if (splits > 1) part = at::empty({B, Hq, splits, D + 2}, q.options().dtype(at::kFloat));
  launch_pdl(kern, dim3(Hkv, B, splits), dim3(128), smem, st, tk, tv, reinterpret_cast<const bf16*>(q.data_ptr()),
             lens.data_ptr<int>(), reinterpret_cast<bf16*>(o.data_ptr()), splits > 1 ? part.data_ptr<float>() : nullptr,
             Hq, lay, scale * kLog2e, splits, err_word(q.device().index()), pf, lead, share_len);
  if (splits > 1) {
    launch_pdl(decode_combine_kernel, dim3(B * Hq), dim3(128), 0, st, part.data_ptr<float>(),
               reinterpret_cast<bf16*>(o.data_ptr()), B * Hq, splits, D);
  }
}

void decode_attn(at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor lens, at::Tensor o, double scale,
                 c10::optional<at::Tensor> prefetch, c10::optional<at::Tensor> lead,
                 c10::optional<at::Tensor> share_len, c10::optional<at::Tensor> block_table) {
  TORCH_CHECK(q.is_contiguous() && kc.is_contiguous() && vc.is_contiguous(), "decode_attn: contiguous");
  TORCH_CHECK(lens.scalar_type() == at::kInt, "decode_attn: int32 lengths");
  if (q.size(0) == 0) return;
  const KvLayout lay = kv_layout_of(kc, block_table);
  TORCH_CHECK(vc.sizes() == kc.sizes() && (lay.table == nullptr ? kc.size(0) == q.size(0)
                                                                 : block_table->size(0) == q.size(0)),
              "decode_attn: cache / block table rows must match the batch");
  const c10::cuda::CUDAGuard g(q.device());
  const int D = static_cast<int>(q.size(2));
  const int rep = static_cast<int>(q.size(1) / kc.size(1));
  const float sc = static_cast<float>(scale);
  const L2Prefetch pf = l2_prefetch_of<L2Prefetch>(prefetch);
  const bool share = lead.has_value() && lead->defined() && share_len.has_value() && share_len->defined();
  if (share) {
    TORCH_CHECK(lead->scalar_type() == at::kInt && share_len->scalar_type() == at::kInt && lead->numel() == q.size(0) &&
                    share_len->numel() == q.size(0) && lead->is_contiguous() && share_len->is_contiguous(),
                "decode_attn: lead / share_len must be int32 [B]");
  }
  const int* ld = share ? lead->data_ptr<int>() : nullptr;
  const int* sl = share ? share_len->data_ptr<int>() : nullptr;
  if (D == 128 && rep == 4) return decode_tc_dispatch<4>(q, kc, vc, lens, o, sc, pf, ld, sl, lay);
  if (D == 128 && rep == 2) return decode_tc_dispatch<2>(q, kc, vc, lens, o, sc, pf, ld, sl, lay);
  if (D == 128 && rep == 8) return decode_tc_dispatch<8>(q, kc, vc, lens, o, sc, pf, ld, sl, lay);
#define VLM_DEC(DD, RR) \
  if (D == DD && rep == RR) return decode_dispatch<DD, RR>(q, kc, vc, lens, o, sc, lay);
  VLM_DEC(128, 4) VLM_DEC(128, 2) VLM_DEC(128, 1) VLM_DEC(128, 8) VLM_DEC(64, 4) VLM_DEC(64, 2) VLM_DEC(64, 1)
  VLM_DEC(32, 2) VLM_DEC(32, 4) VLM_DEC(32, 1)
#undef VLM_DEC
  TORCH_CHECK(false, "decode_attn: unsupported head_dim/group ", D, "/", rep);
}

}  // namespace vlm

// =====================================================================================================
// Allocation-free decode attention entry point.
//
// Declaration: this entry point has no counterpart in the reference project; it exists for callers of
// this library that cannot allocate device memory at call time.  Examples: an inference host whose own
// pool allocator owns all device memory (a cudaMalloc behind its back breaks its accounting and can
// fail under its memory cap), code running where allocation would be an unsynchronised driver call in
// a latency-critical loop, or plugin code that may only touch buffers it was handed.  Such callers
// pass inputs and outputs only; the key-split partial results, which the regular decode_attn path
// keeps in a temporary buffer from the PyTorch allocator, live here in a fixed device array instead,
// and the kernels report a timed-out wait in a second fixed device word rather than in the lazily
// allocated error word of the regular path.  The C declarations are in vlm_noalloc.h.
//
// Contract:
//  * Scratch: the file-scope array below, kNoAllocScratchFloats floats (4 MiB) per GPU.  Every GPU
//    that loads this library holds it until the process exits.  A problem needing more than
//    B * Hq * splits * (D + 2) <= kNoAllocScratchFloats floats is rejected (return value -2).
//  * Set-up: the first call on a device (with that device current) resolves the device addresses of
//    the array and of the status word with cudaGetSymbolAddress; make that first call before any
//    CUDA-graph capture.  Two host threads making their first call at once both resolve the same
//    addresses, so the unsynchronised store of the cached pointer is harmless.
//  * Sharing: all calls on a device share the one array and it keeps the last call's contents.
//    Every partial slot a call reads is written earlier by the same call, unless one of that call's
//    bounded waits ran out, so nothing needs clearing; calls that overlap on the GPU (different
//    streams, or graphs replayed concurrently) race on the array and must be serialised by the caller.
//  * Timeouts: a wait that runs out stops its CTA early and records a non-zero code in the status
//    word; that call's output is then undefined (the merge may read an earlier call's partials).
//    vlmrl_decode_attention_noalloc_status reads and clears the word.
//  * No cudaMalloc, cudaFree or allocating library routine is called, and no C++ exception leaves
//    either function: every failure is a return code.
//  * Return value: 0 ok, -1 unsupported shape, -2 problem exceeds the scratch array, -3 CUDA error.
// =====================================================================================================
namespace vlm {

constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 20;  // 4 MiB of fp32 partials
static __device__ __align__(256) float g_noalloc_decode_scratch[kNoAllocScratchFloats];
static __device__ __align__(16) int g_noalloc_status[4];

namespace {
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlots {
  float* scratch;
  int* status;
};
std::atomic<float*> g_noalloc_scratch_ptr[kNoAllocMaxDevices];
std::atomic<int*> g_noalloc_status_ptr[kNoAllocMaxDevices];

// Device addresses of the scratch array and the status word for the current device, resolved once.
int noalloc_slots(NoAllocSlots& s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return -3;
  s.scratch = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
  s.status = g_noalloc_status_ptr[dev].load(std::memory_order_acquire);
  if (s.scratch && s.status) return 0;
  void* p = nullptr;
  void* w = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_decode_scratch) != cudaSuccess || p == nullptr) return -3;
  if (cudaGetSymbolAddress(&w, g_noalloc_status) != cudaSuccess || w == nullptr) return -3;
  s.scratch = static_cast<float*>(p);
  s.status = static_cast<int*>(w);
  g_noalloc_status_ptr[dev].store(s.status, std::memory_order_release);
  g_noalloc_scratch_ptr[dev].store(s.scratch, std::memory_order_release);
  return 0;
}

template <int D, int REP>
int noalloc_decode_launch(const bf16* q, const bf16* kc, const bf16* vc, const int* lens, bf16* o, int B, int Hq,
                          int Hkv, int Tmax, float scale, const NoAllocSlots& s, int sms, cudaStream_t st) {
  constexpr int NW = 8, KC = 32, STAGES = 4;
  // at least two key splits, so the partial results always go through the scratch array
  const int splits =
      std::max(2, std::min((3 * sms + B * Hkv - 1) / (B * Hkv), std::max(2, Tmax / (2 * KC))));
  if (static_cast<int64_t>(B) * Hq * splits * (D + 2) > kNoAllocScratchFloats) return -2;
  const int smem = 2 * STAGES * KC * D * 2 + STAGES * 8 + (2 * NW * REP + NW * REP * D) * 4;
  auto kern = decode_attn_kernel<D, REP, NW, KC, STAGES>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -3;
  const KvLayout lay{nullptr, 0, Tmax, Hkv, Tmax};  // contiguous [B, Hkv, Tmax, D]
  kern<<<dim3(Hkv, B, splits), NW * 32, smem, st>>>(q, kc, vc, lens, o, s.scratch, Hq, lay, scale * kLog2e, splits,
                                                     s.status);
  if (cudaGetLastError() != cudaSuccess) return -3;
  decode_combine_kernel<<<B * Hq, 128, 0, st>>>(s.scratch, o, B * Hq, splits, D);
  if (cudaGetLastError() != cudaSuccess) return -3;
  return 0;
}

int noalloc_decode(const void* q, const void* k_cache, const void* v_cache, const int* lengths, void* out, int B,
                   int Hq, int Hkv, int Tmax, int D, float scale, void* stream) {
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || Tmax <= 0) return -1;
  const int rep = Hq / Hkv;
  const bool shape_ok = (D == 128 && (rep == 4 || rep == 2 || rep == 1)) || (D == 64 && rep == 4) ||
                        (D == 32 && rep == 2);
  if (!shape_ok) return -1;
  NoAllocSlots s{};
  if (const int rc = noalloc_slots(s)) return rc;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -3;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -3;
  const auto* qq = static_cast<const bf16*>(q);
  const auto* kk = static_cast<const bf16*>(k_cache);
  const auto* vv = static_cast<const bf16*>(v_cache);
  auto* oo = static_cast<bf16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128 && rep == 4) return noalloc_decode_launch<128, 4>(qq, kk, vv, lengths, oo, B, Hq, Hkv, Tmax, scale, s, sms, st);
  if (D == 128 && rep == 2) return noalloc_decode_launch<128, 2>(qq, kk, vv, lengths, oo, B, Hq, Hkv, Tmax, scale, s, sms, st);
  if (D == 128 && rep == 1) return noalloc_decode_launch<128, 1>(qq, kk, vv, lengths, oo, B, Hq, Hkv, Tmax, scale, s, sms, st);
  if (D == 64 && rep == 4) return noalloc_decode_launch<64, 4>(qq, kk, vv, lengths, oo, B, Hq, Hkv, Tmax, scale, s, sms, st);
  return noalloc_decode_launch<32, 2>(qq, kk, vv, lengths, oo, B, Hq, Hkv, Tmax, scale, s, sms, st);
}
}  // namespace

}  // namespace vlm

// q [B, Hq, D] bf16, k_cache / v_cache [B, Hkv, Tmax, D] bf16, lengths [B] int32 (valid keys per
// sequence), out [B, Hq, D] bf16; all device pointers, contiguous.  `stream` is a cudaStream_t (0 for
// the legacy default stream).  Computes out = softmax(q.K^T * scale) . V over the first lengths[b]
// keys of each sequence (grouped-query attention, Hq / Hkv query heads per key head).
extern "C" int vlmrl_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                              const int* lengths, void* out, int B, int Hq, int Hkv, int Tmax, int D,
                                              float scale, void* stream) {
  try {
    return vlm::noalloc_decode(q, k_cache, v_cache, lengths, out, B, Hq, Hkv, Tmax, D, scale, stream);
  } catch (...) {
    return -3;
  }
}

// Waits for `stream`, then stores the status word of the current device in *status (0 = no wait ran
// out since the last read; otherwise the first error code recorded) and clears it.  Returns 0, or -3
// on a CUDA error.
extern "C" int vlmrl_decode_attention_noalloc_status(void* stream, int* status) {
  try {
    vlm::NoAllocSlots s{};
    if (const int rc = vlm::noalloc_slots(s)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    if (cudaMemcpyAsync(&h, s.status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return -3;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -3;
    if (h != 0 && cudaMemsetAsync(s.status, 0, sizeof(int), st) != cudaSuccess) return -3;
    if (status) *status = h;
    return 0;
  } catch (...) {
    return -3;
  }
}
