// Persistent decode step: every decoder layer of one token step of a Qwen3-VL / Qwen2.5-VL text decoder
// (dense, GQA, head_dim 128) in ONE cooperative launch with one CTA per SM.
//
// Why: a decode step at batch <= 128 reads every weight (8 GB for the 4B model) and the KV cache once
// but does little math, so it should run at HBM speed.  As separate kernels (4 GEMMs + 3 consumers +
// attention per layer) every launch pays its pipeline fill and drain.  Here one TMA producer warp per
// SM walks everything the CTA will read from HBM, in consumption order, through one shared-memory ring:
// per layer its share of the qkv weight tiles, the KV-cache chunks of its attention items (the cached
// prefix never depends on the current step), then its o, gate/up and down weight tiles.  The producer
// is throttled only by the ring, never by data dependencies, so HBM keeps streaming while the CTA
// waits for activations.  Reference decode loop: core/sampling.py:157-224 (one jitted step per token).
//
// Per layer (a GEMM unit is a 128-row x 64-k weight tile; CTA c owns units [c*U/Gg, (c+1)*U/Gg) of a GEMM,
// Gg = min(#CTAs, U), walked tile-major, so a tile's k-range is split over a few consecutive CTAs that
// each write an fp32 partial slot):
//   qkv GEMM   -> partials                                  (epilogue warps drain TMEM)
//   attention  : per (sequence, kv-head) item: sum the qkv partials of its REP q heads, k and v, + bias,
//                q/k RMSNorm, RoPE, append k/v to the cache; attention over the ring-staged cached
//                prefix on mma.sync (two 4-warp groups take alternate 64-key chunks), then merge the
//                eight warps' partial softmax states and this step's own key
//   o GEMM     -> partials
//   norm 1     : per (row, 128 columns) warp item: h1 = x + o, partial sum of squares; per-row
//                counter; hn = RMSNorm(h1) * post_norm
//   gate/up    -> partials; the last CTA to finish a tile sums its slots and writes SwiGLU(gate, up)
//   down GEMM  -> partials
//   norm 2     : x = h1 + down, xn = RMSNorm(x) * next layer's input norm (final norm after the last)
// GEMMs are swapped (D^T = W . X^T): the weight tile is the 128-row A operand of tcgen05.mma, the
// activation tile (B rows padded to BP, K-major, 128-byte swizzle) is the N = BP operand, so the MMA is
// never half empty at small batch.  Accumulators are double-buffered in TMEM.
//
// Cross-CTA order: global arrival counters (zeroed before the launch).  A finishing group stores its
// outputs, proxy-fences them for a TMA reader, syncs, fences and increments; a waiter spins on an
// acquire load and fences before its reads or TMA loads.  Every wait is bounded; on expiry the waiter
// raises a global abort word (and the error words) that every other wait polls, the single-thread
// roles drain their copies and MMAs, and every warp still walks its barrier sequence, so the launch
// ends.  All partial sums are added in a fixed order, so a step is bitwise reproducible.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "mma_sync.cuh"

namespace vlm {

using bf16 = __nv_bfloat16;

namespace ds {

constexpr int kThreads = 384;   // warps: 0 ring TMA, 1 MMA, 2 activation TMA, 3 TMEM owner, 4..11 compute
constexpr int kCompute = 256;   // warps 4..11; warps 4..7 are also the TMEM epilogue
constexpr int kTileN = 128;     // weight rows per tile
constexpr int kBK = 64;         // k per stage (128 bytes of bf16, one swizzle row)
constexpr int kSlot = kTileN * kBK * 2;  // ring slot: one weight tile, or one 64-key K or V chunk
constexpr int kD = 128;         // head dim
constexpr int kKC = 64;         // keys per KV chunk
constexpr int kTmemCols = 512;  // two accumulator sets of NA chains x BP columns (NA * BP <= 256)
constexpr long long kWait = 1ll << 31;  // ~1.1 s at 1.9 GHz

// named barriers (0 is __syncthreads)
constexpr int kBarCompute = 1;  // warps 4..11
constexpr int kBarEpi = 2;      // warps 4..7
constexpr int kBarGroup = 3;    // + attention group (0: warps 4..7, 1: warps 8..11)

// sync word layout: the abort word and every phase counter on its own 128-byte line (148 CTAs poll
// them), then the packed per-tile counters of the gate/up last-arriver
constexpr int kAbort = 0;
constexpr int kLine = 32;
constexpr int kCtrPerLayer = 10;
enum Ctr { kQkv = 0, kAtt = 1, kO = 2, kNorm1 = 3, kGuf = 4, kDown = 5, kNorm2 = 6, kNorm1A = 7, kNorm2A = 8 };
constexpr int kMaxItems = 8;    // attention items per CTA: B * Hkv <= 8 * #CTAs

struct Layer {  // 8 pointers (64 bytes), filled by the host from the layer's parameter views
  const bf16* qkv_b;    // may be null
  const bf16* q_norm;   // null: rotation only (no q/k RMSNorm)
  const bf16* k_norm;
  const bf16* post_norm;
  const bf16* next_norm;  // next layer's input norm, or the final norm after the last layer
  bf16* kc;             // [B, Hkv, Tmax, D] cache slice of this layer
  bf16* vc;
  const void* pad;
};

struct Params {
  int L, B, BP, H, nq, nkv, F, Tmax, G;
  int NA;  // independent MMA accumulation chains per tile: k-step i of a k-block accumulates into chain i % NA
  int w_stages, slot_bytes;  // ring slots: a 16 KB weight tile / KV chunk, then the k-block's activation tile
  float eps, scale_log2;
  const CUtensorMap* wmaps;  // [L][4] weights (qkv, o, gate/up, down; [N, K] row-major), then [L][2] K / V caches
  const CUtensorMap* amaps;  // [4]: xn, o, hn, act activations ([B, K] row-major)
  const Layer* layers;
  bf16* x;    // [B, H] residual stream (in: embedded tokens; out: last layer's residual)
  bf16* h1;   // [B, H]
  bf16* xn;   // [B, H] (in: normed input of layer 0; out: final-normed hidden)
  bf16* o;    // [B, nq * D]
  bf16* hn;   // [B, H]
  bf16* act;  // [B, F]
  float* ws;  // fp32 partial slots
  float* ssq; // [2][B][H / 128] partial sums of squares of the two norms
  const int* lens;
  const int64_t* delta;
  const float* inv_freq;  // [D / 2]
  const int* lead;        // may be null
  const int* share_len;
  unsigned* sync;
  int* err;
  long long* trace;  // optional [G][L][16] globaltimer stamps (ns) of phase boundaries, null = off
};

// A GEMM's units are spread over Gg = min(G, U) CTAs, so every participating CTA owns at least one unit
// and the CTAs touching a tile are consecutive: slot = CTA - first CTA of the tile, no gaps.
struct Gemm {
  int N, K, T, KB, Gg, U;  // U <= 192 tiles x 192 k-blocks: 32-bit index math throughout
};

VLM_DEV Gemm gemm_of(const Params& p, int g) {
  Gemm m;
  const int qkv = (p.nq + 2 * p.nkv) * kD;
  m.N = g == 0 ? qkv : g == 1 ? p.H : g == 2 ? 2 * p.F : p.H;
  m.K = g == 0 ? p.H : g == 1 ? p.nq * kD : g == 2 ? p.H : p.F;
  m.T = m.N / kTileN;
  m.KB = m.K / kBK;
  m.U = m.T * m.KB;
  m.Gg = m.U < p.G ? m.U : p.G;
  return m;
}
VLM_DEV int unit_begin(const Gemm& m, int c) { return c >= m.Gg ? m.U : m.U * c / m.Gg; }
// CTA that owns unit u
VLM_DEV int cta_of(const Gemm& m, int u) { return ((u + 1) * m.Gg - 1) / m.U; }
VLM_DEV int slots_of(const Gemm& m, int tile) {
  const int first = tile * m.KB;
  return cta_of(m, first + m.KB - 1) - cta_of(m, first) + 1;
}

// Attention item (sequence b, kv head hk): its cached prefix [0, len) in 64-key chunks, the shared-prompt
// part [0, s) read from the group leader's row and the rest from row b, chunks never straddling s.
struct Item {
  int b, hk, len, s, lead, n_shared, n_chunks;
};
VLM_DEV Item item_of(const Params& p, int item) {
  Item it;
  it.b = item / p.nkv;
  it.hk = item - it.b * p.nkv;
  it.len = min(p.lens[it.b], p.Tmax - 1);
  it.lead = p.lead ? p.lead[it.b] : it.b;
  it.s = p.share_len ? min(p.share_len[it.b], it.len) : 0;
  if (it.lead == it.b) it.s = 0;
  it.n_shared = (it.s + kKC - 1) / kKC;
  it.n_chunks = it.n_shared + (it.len - it.s + kKC - 1) / kKC;
  return it;
}
// chunk j of an item: first key, number of keys and the cache row it is read from
VLM_DEV void chunk_of(const Item& it, int j, int& k0, int& cnt, int& row) {
  if (j < it.n_shared) {
    k0 = j * kKC;
    cnt = min(kKC, it.s - k0);
    row = it.lead;
  } else {
    k0 = it.s + (j - it.n_shared) * kKC;
    cnt = min(kKC, it.len - k0);
    row = it.b;
  }
}
// ring slots this CTA's attention items occupy in one layer (K and V per chunk)
VLM_DEV int kv_slots(const Params& p, int c) {
  int n = 0;
  for (int item = c; item < p.B * p.nkv; item += p.G) n += 2 * item_of(p, item).n_chunks;
  return n;
}

// Phase-boundary timestamps for latency analysis (VLMRL_DS_TRACE=1 on the host side).
enum TraceEv {
  kTrQkvEpi = 0, kTrQkvWait, kTrAtt, kTrOEpi, kTrOWait, kTrNorm1, kTrGuEpi, kTrDownEpi, kTrDownWait, kTrNorm2,
  kTrMmaQkv, kTrMmaO, kTrMmaGu, kTrMmaDown, kTrWQkv, kTrWGu
};
VLM_DEV void trace(const Params& p, int layer, int ev) {
  if (p.trace == nullptr) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  p.trace[(static_cast<long long>(blockIdx.x) * p.L + layer) * 16 + ev] = static_cast<long long>(t);
}

// Per-CTA wait statistics (cycles), in the trace buffer's extra row [G][L][16] + c * 16 + stat.
enum Stat {
  kStProdGemm = 0, kStProdKv, kStMmaW, kStMmaA, kStMmaT, kStActCtr, kStActEmpty, kStAttKv, kStEpiT, kStTotal,
  kStGroupWait, kStAttention, kStNorm, kStQkvConsume
};
// Accumulated in shared memory (flushed to the trace buffer once at exit), so a wait costs no global atomic.
__shared__ unsigned long long ds_stats[16];
VLM_DEV void stat_add(const Params& p, int stat, long long cycles) {
  if (p.trace == nullptr || (threadIdx.x & 31) != 0) return;
  atomicAdd(&ds_stats[stat], static_cast<unsigned long long>(cycles));
}
// Event log of CTA 0, layer 1 (trace on): [stream][k-block] globaltimer ns after the stats block;
// stream 0 = activation TMA issued, 1 = MMA saw the activation tile, 2 = MMA saw the weight tile,
// 3 = weight tile issued.
VLM_DEV void evlog(const Params& p, int layer, int stream, int idx) {
  if (p.trace == nullptr || blockIdx.x != 0 || layer != 1 || idx >= 256) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  p.trace[static_cast<long long>(p.G) * (p.L + 1) * 16 + stream * 256 + idx] = static_cast<long long>(t);
}
// timed(p, stat, expr): evaluates expr and, with tracing on, adds the cycles it took to the CTA's stat.
#define DS_TIMED(p, stat, expr)                                  \
  ([&]() {                                                       \
    const long long t0_ = (p).trace ? clock64() : 0;             \
    auto r_ = (expr);                                            \
    if ((p).trace) stat_add((p), (stat), clock64() - t0_);       \
    return r_;                                                   \
  }())

VLM_DEV unsigned* ctr(const Params& p, int layer, int which) {
  return p.sync + (1 + layer * kCtrPerLayer + which) * kLine;
}
VLM_DEV unsigned* tile_ctr(const Params& p, int layer, int tile, int T) {
  return p.sync + (1 + p.L * kCtrPerLayer) * kLine + layer * T + tile;
}

VLM_DEV bool aborted(const Params& p) { return *reinterpret_cast<volatile unsigned*>(p.sync + kAbort) != 0u; }
// The first waiter to give up records its code, CTA and the wait it gave up on in the error words.
VLM_DEV void ds_raise(const Params& p, int code, int where = -1) {
  atomicExch(p.sync + kAbort, 1u);
  if (atomicCAS(p.err, 0, code) == 0) {
    p.err[1] = blockIdx.x;
    p.err[2] = where;
  }
}
VLM_DEV unsigned ld_acquire(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
VLM_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
VLM_DEV void bar_named(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Bounded mbarrier wait that also gives up when another CTA raised the abort word.
VLM_DEV bool mwait(uint64_t* bar, uint32_t parity, const Params& p, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (int it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (aborted(p)) return false;
      if (clock64() - t0 > kWait) {
        ds_raise(p, code, -2);
        return false;
      }
    }
  }
}
// Warp-wide wait with a single polling lane; the result is broadcast, so the warp takes one path.
VLM_DEV bool mwait_warp(uint64_t* bar, uint32_t parity, const Params& p, int code) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mwait(bar, parity, p, code);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}
// Bounded wait (no abort polling) used only to drain this CTA's own copies / MMAs before it exits.
VLM_DEV void mwait_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity) && clock64() - t0 < kWait) {
  }
}
VLM_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// One thread: wait until *c >= target (acquire), bounded, abort-aware.
VLM_DEV bool cwait(const Params& p, const unsigned* c, unsigned target, int code) {
  const long long t0 = clock64();
  while (true) {
    const unsigned v = ld_acquire(c);
    if (v >= target) return true;
    if (aborted(p)) return false;
    if (clock64() - t0 > kWait) {
      ds_raise(p, code, static_cast<int>(c - p.sync));
      p.err[3] = static_cast<int>(v);
      return false;
    }
    __nanosleep(20);
  }
}
// One thread after its group synced: release the group's stores, then count.
VLM_DEV void arrive(unsigned* c) {
  fence_acq_rel_gpu();
  atomicAdd(c, 1u);
}

VLM_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
VLM_DEV void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}
// Sum of `slots` partial float4s at base + s * stride, s = 0..slots-1 in order; the first MAXS loads are
// all issued before the first add (MAXS is sized per call site to the slot counts its GEMM produces).
template <int MAXS>
VLM_DEV float4 sum_slots4(const float* base, long long stride, int slots) {
  float4 v[MAXS];
#pragma unroll
  for (int i = 0; i < MAXS; ++i)
    if (i < slots) v[i] = ldcg4(base + i * stride);
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < MAXS; ++i)
    if (i < slots) add4(a, v[i]);
  for (int i = MAXS; i < slots; ++i) add4(a, ldcg4(base + i * stride));
  return a;
}

// 64-column bf16 tile with the 128-byte TMA swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7).
VLM_DEV int sw64(int row, int col) { return row * 64 + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7); }
// mma.sync B fragments for two n-blocks (n0, n0 + 8) x one k-step from a tile stored [n][k] / [k][n].
VLM_DEV void frag_nk(uint32_t (&b)[4], const bf16* s, int n0, int k0, int lane) {
  const int r = n0 + (lane & 7) + (lane >> 4) * 8;
  const int c = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(b, s + sw64(r, c));
}
VLM_DEV void frag_kn(uint32_t (&b)[4], const bf16* s, int k0, int n0, int lane) {
  const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = n0 + (lane >> 4) * 8;
  ldsm_x4_t(b, s + sw64(r, c));
}

struct Smem {
  uint8_t* wbuf;     // the ring: w_stages slots of slot_bytes (weight tile or KV chunk, then activation tile)
  float* merge;      // [8 warps][REP][D + 2]
  bf16* qs;          // [kMaxItems][REP][D] the items' rotated q heads
  bf16* kvn;         // [kMaxItems][2][D] the items' k and v of this step
  float* red;        // [16]
  uint64_t* wfull;   // two arrivals: the ring producer's and the activation producer's
  uint64_t* wempty;
  uint64_t* tfull;   // [2]
  uint64_t* tempty;  // [2]
  uint64_t* drain;
  uint64_t* kvdone;  // one arrival per layer: the attention warps are done with the layer's KV slots
  uint32_t* tmem_holder;
  int* flags;        // [0] compute-group wait result, [1] last-arriver flag
};

__host__ __device__ inline int a_stage_bytes(int BP) { return BP * kBK * 2; }
// the attention merge area [8 warps][REP][D + 2], also the norms' staging of h [8 warps][4 items][128]
__host__ __device__ inline int merge_floats(int rep) {
  return 8 * rep * (kD + 2) > 8 * 4 * kTileN ? 8 * rep * (kD + 2) : 8 * 4 * kTileN;
}

// ------------------------------------------------------------------ epilogue of one GEMM phase
// Warps 4..7: drain this CTA's accumulator segments of GEMM g into fp32 partial slots ws[slot][b][n];
// for gate/up the last CTA to finish a tile writes act = SwiGLU over the tile's 64 columns.
VLM_DEV void epilogue_phase(const Params& p, const Smem& s, uint32_t tmem_base, int layer, int g, int& lt) {
  const Gemm m = gemm_of(p, g);
  const int c = blockIdx.x;
  const int et = threadIdx.x - 128;  // 0..127
  const int q = (threadIdx.x >> 5) & 3;
  const int lane = threadIdx.x & 31;
  int u = unit_begin(m, c);
  const int u1 = unit_begin(m, c + 1);
  while (u < u1) {
    const int tile = u / m.KB;
    const int kb0 = u - tile * m.KB;
    const int kb1 = min(m.KB, kb0 + (u1 - u));
    u += kb1 - kb0;
    const int slot = c - cta_of(m, tile * m.KB);
    const int acc = lt & 1;
    const uint32_t use = static_cast<uint32_t>(lt >> 1);
    ++lt;
    // warp-uniform: tcgen05.ld below is .sync.aligned
    const bool ok = et == 0 ? DS_TIMED(p, kStEpiT, mwait_warp(&s.tfull[acc], use & 1u, p, kErrTimeoutEpilogue))
                            : mwait_warp(&s.tfull[acc], use & 1u, p, kErrTimeoutEpilogue);
    tc_fence_after();
    if (ok) {
      const int n = tile * kTileN + q * 32 + lane;
      float* dst = p.ws + static_cast<long long>(slot) * p.B * m.N + n;
      const uint32_t tb =
          tmem_base + static_cast<uint32_t>(acc * p.NA * p.BP) + (static_cast<uint32_t>(q * 32) << 16);
      for (int j = 0; j < p.BP / 16; ++j) {
        float v[16];
        uint32_t r[16];
        tmem_ld16(tb + j * 16, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(r[e]);
        for (int ch = 1; ch < p.NA; ++ch) {  // the chains in a fixed order
          tmem_ld16(tb + ch * p.BP + j * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] += __uint_as_float(r[e]);
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int b = j * 16 + e;
          if (b < p.B) dst[static_cast<long long>(b) * m.N] = v[e];
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.tempty[acc]);
    if (g == 2) {
      // last arriver of the tile finishes SwiGLU for its 64 activation columns
      bar_named(kBarEpi, 128);
      if (et == 0) {
        fence_acq_rel_gpu();
        const int slots = slots_of(m, tile);
        const unsigned old = atomicAdd(tile_ctr(p, layer, tile, m.T), 1u);
        s.flags[1] = (old == static_cast<unsigned>(slots - 1)) ? 1 : 0;
        fence_acq_rel_gpu();
      }
      bar_named(kBarEpi, 128);
      if (s.flags[1]) {
        const int slots = slots_of(m, tile);
        const long long stride = static_cast<long long>(p.B) * m.N;
        for (int it = et; it < p.B * 16; it += 128) {
          const int b = it >> 4, c4 = it & 15;
          const int col = tile * kTileN + c4 * 8;  // 8 gate/up columns -> 4 activation columns
          const float* src = p.ws + static_cast<long long>(b) * m.N + col;
          const float4 v0 = sum_slots4<3>(src, stride, slots);
          const float4 v1 = sum_slots4<3>(src + 4, stride, slots);
          const float gv[4] = {v0.x, v0.z, v1.x, v1.z}, uv[4] = {v0.y, v0.w, v1.y, v1.w};
          float o4[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float gg = bf2f(f2bf(gv[j])), uu = bf2f(f2bf(uv[j]));
            o4[j] = gg / (1.f + __expf(-gg)) * uu;
          }
          *reinterpret_cast<uint2*>(p.act + static_cast<long long>(b) * p.F + tile * 64 + c4 * 4) =
              make_uint2(pack_bf16x2(o4[0], o4[1]), pack_bf16x2(o4[2], o4[3]));
        }
        fence_proxy_async_global();
        bar_named(kBarEpi, 128);
        if (et == 0) arrive(ctr(p, layer, kGuf));
      }
    }
  }
  if (g != 2) {
    fence_proxy_async_global();
    bar_named(kBarEpi, 128);
    if (et == 0) arrive(ctr(p, layer, g == 0 ? kQkv : g == 1 ? kO : kDown));
  }
}

// All compute warps wait until *c >= target; the result is shared so every warp takes the same path.
VLM_DEV bool group_wait(const Params& p, const Smem& s, const unsigned* c, unsigned target, int code) {
  const int ct = threadIdx.x - 128;
  if (ct == 0) s.flags[0] = DS_TIMED(p, kStGroupWait, cwait(p, c, target, code)) ? 1 : 0;
  bar_named(kBarCompute, kCompute);
  const bool ok = s.flags[0] != 0;
  bar_named(kBarCompute, kCompute);  // flags[0] is rewritten by the next wait only after everyone read it
  return ok;
}
// tma_reader: the stores being released are read next by TMA (async proxy), so order them for it first.
VLM_DEV void group_arrive(const Params& p, unsigned* c, bool tma_reader = true) {
  if (tma_reader) fence_proxy_async_global();
  bar_named(kBarCompute, kCompute);
  if (threadIdx.x == 128) arrive(c);
}

// ------------------------------------------------------------------ attention (+ q/k/v consumer)
// rp: ring position of this layer's first KV slot for this CTA.
template <int REP>
VLM_DEV void attention_phase(const Params& p, const Smem& s, int layer, int rp) {
  const Layer& ly = p.layers[layer];
  const Gemm m = gemm_of(p, 0);
  const int ct = threadIdx.x - 128, cw = ct >> 5, lane = ct & 31;
  const int grp = cw >> 2, wg = cw & 3;  // attention group and warp in group
  const int g = lane >> 2, tq = lane & 3;
  const int S = p.w_stages;
  const long long stride = static_cast<long long>(p.B) * m.N;
  // ---- 1) for every item of this CTA: its REP q heads, k and v from the qkv partials (+ bias, q/k RMSNorm,
  // RoPE; k / v appended to the cache), all loads of a warp's heads in flight together
  const int n_items = (p.B * p.nkv - blockIdx.x + p.G - 1) / p.G;
  for (int pr = cw; pr < n_items * (REP + 2); pr += 8) {
    const int ii = pr / (REP + 2), hh = pr - ii * (REP + 2);
    const Item it = item_of(p, blockIdx.x + ii * p.G);
    const int b = it.b, hk = it.hk, len = it.len;
    {
      const int head = hh < REP ? hk * REP + hh : (hh == REP ? p.nq + hk : p.nq + p.nkv + hk);
      const int d0 = lane * 4;
      const bool is_q = hh < REP, is_v = hh == REP + 1;
      const bf16* nw = is_q ? ly.q_norm : ly.k_norm;
      // independent loads first: bias, norm weight, rotary frequencies, position offset, partial slots
      const uint2 bias = ly.qkv_b ? *reinterpret_cast<const uint2*>(ly.qkv_b + head * kD + d0) : make_uint2(0, 0);
      const uint2 nwv = (!is_v && nw) ? *reinterpret_cast<const uint2*>(nw + d0) : make_uint2(0, 0);
      const float4 fr = *reinterpret_cast<const float4*>(p.inv_freq + (d0 & 63));
      const long long dl = p.delta[b];
      const float4 sum =
          sum_slots4<6>(p.ws + static_cast<long long>(b) * m.N + head * kD + d0, stride, slots_of(m, head));
      const float2 b01 = unpack_bf16x2(bias.x), b23 = unpack_bf16x2(bias.y);
      float x[4] = {bf2f(f2bf(sum.x + b01.x)), bf2f(f2bf(sum.y + b01.y)), bf2f(f2bf(sum.z + b23.x)),
                    bf2f(f2bf(sum.w + b23.y))};
      const long long cache_off = ((static_cast<long long>(b) * p.nkv + hk) * p.Tmax + len) * kD + d0;
      bf16* kvn = s.kvn + ii * 2 * kD;
      if (is_v) {  // v: appended as is
        const uint2 pk = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
        *reinterpret_cast<uint2*>(ly.vc + cache_off) = pk;
        *reinterpret_cast<uint2*>(kvn + kD + d0) = pk;
        continue;
      }
      float r = 1.f;
      if (nw) {
        float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
        ss = warp_sum(ss);
        r = rsqrtf(ss / kD + p.eps);
      }
      const float2 n01 = unpack_bf16x2(nwv.x), n23 = unpack_bf16x2(nwv.y);
      const float nwf[4] = {n01.x, n01.y, n23.x, n23.y};
      const float frf[4] = {fr.x, fr.y, fr.z, fr.w};
      float xn[4], y[4], out[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xn[i] = nw ? x[i] * r * nwf[i] : x[i];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = __shfl_xor_sync(0xffffffffu, xn[i], 16);  // dims d -+ 64
      const float pos = static_cast<float>(static_cast<long long>(len) + dl);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float sn, cs;
        sincosf(pos * frf[i], &sn, &cs);
        out[i] = d0 < 64 ? xn[i] * cs - y[i] * sn : xn[i] * cs + y[i] * sn;
      }
      const uint2 pk = make_uint2(pack_bf16x2(out[0], out[1]), pack_bf16x2(out[2], out[3]));
      if (is_q) {
        *reinterpret_cast<uint2*>(s.qs + (ii * REP + hh) * kD + d0) = pk;
      } else {
        *reinterpret_cast<uint2*>(ly.kc + cache_off) = pk;
        *reinterpret_cast<uint2*>(kvn + d0) = pk;
      }
    }
  }
  bar_named(kBarCompute, kCompute);  // q, k and v of every item in shared memory
  int cbase = 0;  // KV chunks of this layer's earlier items
  for (int ii = 0; ii < n_items; ++ii) {
    const Item it = item_of(p, blockIdx.x + ii * p.G);
    const int b = it.b, hk = it.hk;
    const bf16* qs = s.qs + ii * REP * kD;
    const bf16* kvn = s.kvn + ii * 2 * kD;
    // ---- 2) the cached prefix: group grp takes the chunks whose index among the layer's chunks has parity
    // grp (K in ring position rp + 2j, V in rp + 2j + 1).  A parity wait on a slot is only exact when the
    // slot's previous phase is already complete; the ring depth is a multiple of 4, so that previous phase
    // (S positions back = S / 2 chunks back, an even count) is a chunk this group has waited on itself.
    uint32_t qa[kD / 16][4];
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk) {
      qa[kk][1] = qa[kk][3] = 0u;
      if (g < REP) {
        const bf16* qr = qs + g * kD + kk * 16 + 2 * tq;
        qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr);
        qa[kk][2] = *reinterpret_cast<const uint32_t*>(qr + 8);
      } else {
        qa[kk][0] = qa[kk][2] = 0u;
      }
    }
    float acc[kD / 8][4];
#pragma unroll
    for (int i = 0; i < kD / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;  // running stats of row g (rows g < REP are the heads)
    for (int j = grp ^ (cbase & 1); j < it.n_chunks; j += 2) {
      int k0, cnt, row;
      chunk_of(it, j, k0, cnt, row);
      const int pk = rp + 2 * j, pv = pk + 1;
      const bool okk = DS_TIMED(p, kStAttKv, mwait_warp(&s.wfull[pk % S], static_cast<uint32_t>((pk / S) & 1), p, kErrTimeoutFlag));
      const bool okv = mwait_warp(&s.wfull[pv % S], static_cast<uint32_t>((pv / S) & 1), p, kErrTimeoutFlag);
      const bf16* kt = reinterpret_cast<const bf16*>(s.wbuf + (pk % S) * p.slot_bytes);
      bf16* vt = reinterpret_cast<bf16*>(s.wbuf + (pv % S) * p.slot_bytes);
      if (okk && okv) {
        if (cnt < kKC) {
          // keys past the chunk's range: their V rows hold another sequence's or unwritten cache rows, and
          // P = 0 does not cancel a NaN there, so zero this warp's invalid rows before P.V reads them
          for (int i = lane; i < 16 * 16; i += 32) {
            const int r = wg * 16 + (i >> 4), chn = i & 15;
            if (r >= cnt) reinterpret_cast<uint4*>(vt + (chn >> 3) * (kKC * 64) + r * 64)[chn & 7] = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();  // the next TMA write to this slot is ordered after these stores
          __syncwarp();
        }
        float sc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          uint32_t bb[4];
          frag_nk(bb, kt + (kk >> 2) * (kKC * 64), wg * 16, (kk & 3) * 16, lane);
          mma_bf16(sc[0], qa[kk], bb[0], bb[1]);
          mma_bf16(sc[1], qa[kk], bb[2], bb[3]);
        }
        float mx = -INFINITY;
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool ok = wg * 16 + nb * 8 + 2 * tq + e < cnt;
            sc[nb][e] = ok ? sc[nb][e] * p.scale_log2 : -INFINITY;
            mx = fmaxf(mx, sc[nb][e]);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(mrun, mx);
        const float base = mn == -INFINITY ? 0.f : mn;
        const float cf = exp2f(mrun - base);
        float ps = 0.f;
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            sc[nb][e] = exp2f(sc[nb][e] - base);
            ps += sc[nb][e];
          }
        lrun = lrun * cf + ps;
        mrun = mn;
#pragma unroll
        for (int i = 0; i < kD / 8; ++i) {
          acc[i][0] *= cf;
          acc[i][1] *= cf;
        }
        uint32_t pa[4];
        pa[0] = pack_bf16x2(sc[0][0], sc[0][1]);
        pa[1] = 0u;
        pa[2] = pack_bf16x2(sc[1][0], sc[1][1]);
        pa[3] = 0u;
#pragma unroll
        for (int dp = 0; dp < kD / 16; ++dp) {
          uint32_t bb[4];
          frag_kn(bb, vt + (dp >> 2) * (kKC * 64), wg * 16, (dp & 3) * 16, lane);
          mma_bf16(acc[2 * dp], pa, bb[0], bb[1]);
          mma_bf16(acc[2 * dp + 1], pa, bb[2], bb[3]);
        }
      }
      bar_named(kBarGroup + grp, 128);  // the group is done with both slots
      if (wg == 0 && lane == 0) {
        mbar_arrive(&s.wempty[pk % S]);
        mbar_arrive(&s.wempty[pv % S]);
      }
    }
    rp += 2 * it.n_chunks;
    cbase += it.n_chunks;
    // ---- 3) merge the eight warps' states and this step's own key
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    float* mw = s.merge + cw * REP * (kD + 2);
    if (g < REP) {
      float* row = mw + g * (kD + 2);
      if (tq == 0) {
        row[0] = mrun;
        row[1] = lrun;
      }
#pragma unroll
      for (int nb = 0; nb < kD / 8; ++nb) {
        row[2 + nb * 8 + 2 * tq] = acc[nb][0];
        row[2 + nb * 8 + 2 * tq + 1] = acc[nb][1];
      }
    }
    if (cw < REP) {  // score of this step's own key for head cw
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) d += bf2f(qs[cw * kD + lane * 4 + i]) * bf2f(kvn[lane * 4 + i]);
      d = warp_sum(d);
      if (lane == 0) s.red[cw] = d * p.scale_log2;
    }
    bar_named(kBarCompute, kCompute);
    for (int i = ct; i < REP * kD; i += kCompute) {
      const int r = i / kD, d = i - r * kD;
      const float sn = s.red[r];
      float mxx = sn;
#pragma unroll
      for (int w = 0; w < 8; ++w) mxx = fmaxf(mxx, s.merge[(w * REP + r) * (kD + 2)]);
      float lt = exp2f(sn - mxx), at = lt * bf2f(kvn[kD + d]);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float* e = s.merge + (w * REP + r) * (kD + 2);
        const float cfw = e[0] == -INFINITY ? 0.f : exp2f(e[0] - mxx);
        lt += e[1] * cfw;
        at += e[2 + d] * cfw;
      }
      p.o[static_cast<long long>(b) * p.nq * kD + (hk * REP + r) * kD + d] = f2bf(at / lt);
    }
    bar_named(kBarCompute, kCompute);  // the merge area is reused by the next item
  }
}

// ------------------------------------------------------------------ residual + RMSNorm
// Work items are (row b, 128-column tile t), one per warp over every CTA.  Pass A: h = res + partials
// (bf16) and a per-(row, tile) partial sum of squares.  A grid counter, then pass B: the row's sum of
// squares from its partials in tile order, out = RMSNorm(h) * w.
// second == false: res = x, h -> h1, out -> hn (post_norm);  second == true: res = h1, h -> x, out -> xn.
VLM_DEV void norm_phase(const Params& p, const Smem& s, int layer, bool second) {
  const Layer& ly = p.layers[layer];
  const Gemm m = gemm_of(p, second ? 3 : 1);
  const int ct = threadIdx.x - 128, cw = ct >> 5, lane = ct & 31;
  const int H = p.H, T = H / kTileN;
  const bf16* res_in = second ? p.h1 : p.x;
  bf16* h_out = second ? p.x : p.h1;
  bf16* n_out = second ? p.xn : p.hn;
  const bf16* w = second ? ly.next_norm : ly.post_norm;
  float* ssq = p.ssq + (second ? p.B * T : 0);
  const int nwarps = p.G * 8;
  const int wid = blockIdx.x * 8 + cw;
  const long long stride = static_cast<long long>(p.B) * m.N;
  const int items = p.B * T;
  constexpr int kNormItems = 4;
  // a warp owns at most kNormItems items (B * H / 128 <= kNormItems * 8 * #CTAs); their h values wait in the
  // attention merge area (idle during the norms) across the grid counter
  float* hs = s.merge + (cw * kNormItems) * kTileN;
#pragma unroll 1
  for (int k = 0; k < kNormItems; ++k) {
    const int item = wid + k * nwarps;
    if (item >= items) break;
    const int b = item / T, t = item - b * T;
    const int col = t * kTileN + lane * 4;
    const uint2 rv = __ldcg(reinterpret_cast<const uint2*>(res_in + static_cast<long long>(b) * H + col));
    const float4 v = sum_slots4<10>(p.ws + static_cast<long long>(b) * m.N + col, stride, slots_of(m, t));
    const float2 r0 = unpack_bf16x2(rv.x), r1 = unpack_bf16x2(rv.y);
    const float4 h = make_float4(bf2f(f2bf(v.x + r0.x)), bf2f(f2bf(v.y + r0.y)), bf2f(f2bf(v.z + r1.x)),
                                 bf2f(f2bf(v.w + r1.y)));
    *reinterpret_cast<uint2*>(h_out + static_cast<long long>(b) * H + col) =
        make_uint2(pack_bf16x2(h.x, h.y), pack_bf16x2(h.z, h.w));
    *reinterpret_cast<float4*>(hs + k * kTileN + lane * 4) = h;
    const float ss = warp_sum(h.x * h.x + h.y * h.y + h.z * h.z + h.w * h.w);
    if (lane == 0) ssq[b * T + t] = ss;
  }
  unsigned* ca = ctr(p, layer, second ? kNorm2A : kNorm1A);
  group_arrive(p, ca, false);
  group_wait(p, s, ca, static_cast<unsigned>(p.G), kErrTimeoutFlag);
#pragma unroll 1
  for (int k = 0; k < kNormItems; ++k) {
    const int item = wid + k * nwarps;
    if (item >= items) break;
    const int b = item / T, t = item - b * T;
    const int col = t * kTileN + lane * 4;
    const uint2 wv = *reinterpret_cast<const uint2*>(w + col);
    float tot = 0.f;
    for (int i = lane; i < T; i += 32) tot += __ldcg(ssq + b * T + i);
    tot = warp_sum(tot);
    const float r = rsqrtf(tot / H + p.eps);
    const float4 h = *reinterpret_cast<const float4*>(hs + k * kTileN + lane * 4);
    const float2 w0 = unpack_bf16x2(wv.x), w1 = unpack_bf16x2(wv.y);
    const float o0 = bf2f(f2bf(h.x * r)) * w0.x, o1 = bf2f(f2bf(h.y * r)) * w0.y;
    const float o2 = bf2f(f2bf(h.z * r)) * w1.x, o3 = bf2f(f2bf(h.w * r)) * w1.y;
    *reinterpret_cast<uint2*>(n_out + static_cast<long long>(b) * H + col) =
        make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
}

// ------------------------------------------------------------------ the kernel
template <int REP>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t ds_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ds_raw) + 1023) & ~uintptr_t(1023));
  const int abytes = a_stage_bytes(p.BP);
  const int SB = p.slot_bytes;
  Smem s;
  s.wbuf = base;
  s.merge = reinterpret_cast<float*>(s.wbuf + p.w_stages * SB);
  s.qs = reinterpret_cast<bf16*>(s.merge + merge_floats(REP));
  s.kvn = s.qs + kMaxItems * REP * kD;
  s.red = reinterpret_cast<float*>(s.kvn + kMaxItems * 2 * kD);
  s.wfull = reinterpret_cast<uint64_t*>(s.red + 16);
  s.wempty = s.wfull + p.w_stages;
  s.tfull = s.wempty + p.w_stages;
  s.tempty = s.tfull + 2;
  s.drain = s.tempty + 2;
  s.kvdone = s.drain + 1;
  s.tmem_holder = reinterpret_cast<uint32_t*>(s.kvdone + 1);
  s.flags = reinterpret_cast<int*>(s.tmem_holder + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < 16) ds_stats[threadIdx.x] = 0ull;
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.w_stages; ++i) {
      mbar_init(&s.wfull[i], 2);
      mbar_init(&s.wempty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&s.tfull[a], 1);
      mbar_init(&s.tempty[a], 4);
    }
    mbar_init(s.drain, 1);
    mbar_init(s.kvdone, 1);
    s.flags[0] = s.flags[1] = 0;
    fence_mbar_init();
  }
  if (warp == 3) {
    tmem_alloc(s.tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_holder;
  const int c = blockIdx.x;
  const long long t_start = clock64();

  if (warp == 0) {
    // ---- ring producer: per layer the qkv tiles, the KV chunks of this CTA's items, o, gate/up, down.  The
    // whole warp walks the loop (no lane parks at a CTA barrier); lane 0 issues.
    int st = 0;
    uint32_t ph = 0;
    long long issued = 0;
    bool ok = true;
    auto advance = [&]() {
      ++issued;
      if (++st == p.w_stages) {
        st = 0;
        ph ^= 1u;
      }
    };
    for (int layer = 0; ok && layer < p.L; ++layer) {
      int wlog = 0;
      for (int g = 0; ok && g < 4; ++g) {
        const Gemm m = gemm_of(p, g);
        const CUtensorMap* map = p.wmaps + layer * 4 + g;
        const int u0 = unit_begin(m, c), u1 = unit_begin(m, c + 1);
        int tile = u0 / m.KB, kb = u0 - tile * m.KB;  // walked incrementally: no division per tile
        if (u0 < u1 && (g == 0 || g == 2)) trace(p, layer, g == 0 ? kTrWQkv : kTrWGu);
        for (int u = u0; u < u1; ++u) {
          if (!DS_TIMED(p, kStProdGemm, mwait_warp(&s.wempty[st], ph ^ 1u, p, kErrTimeoutProducer))) {
            ok = false;
            break;
          }
          if (lane == 0) {
            evlog(p, layer, 3, wlog++);
            mbar_arrive_expect_tx(&s.wfull[st], kSlot);
            tma_load_2d(s.wbuf + st * SB, map, &s.wfull[st], kb * kBK, tile * kTileN);
          }
          __syncwarp();
          advance();
          if (++kb == m.KB) {
            kb = 0;
            ++tile;
          }
        }
        if (g != 0) continue;
        // the cached prefix of this CTA's attention items: per chunk a K slot and a V slot, each two
        // 64 x 64 boxes of the [B * Hkv * Tmax, D] cache view
        const CUtensorMap* kmap = p.wmaps + p.L * 4 + layer * 2;
        for (int item = c; ok && item < p.B * p.nkv; item += p.G) {
          const Item it = item_of(p, item);
          for (int j = 0; ok && j < it.n_chunks; ++j) {
            int k0, cnt, row;
            chunk_of(it, j, k0, cnt, row);
            const int y = (row * p.nkv + it.hk) * p.Tmax + k0;
            for (int kv = 0; kv < 2; ++kv) {
              if (!DS_TIMED(p, kStProdKv, mwait_warp(&s.wempty[st], ph ^ 1u, p, kErrTimeoutProducer))) {
                ok = false;
                break;
              }
              if (lane == 0) {
                mbar_arrive_expect_tx(&s.wfull[st], kSlot);
                uint8_t* dst = s.wbuf + st * SB;
                tma_load_2d(dst, kmap + kv, &s.wfull[st], 0, y);
                tma_load_2d(dst + kSlot / 2, kmap + kv, &s.wfull[st], 64, y);
              }
              __syncwarp();
              advance();
            }
          }
        }
      }
    }
    // every copy this warp issued has landed before the CTA can exit (also when a consumer gave up)
    for (long long i = issued - 1; i >= 0 && i >= issued - p.w_stages; --i)
      mwait_drain(&s.wfull[i % p.w_stages], static_cast<uint32_t>((i / p.w_stages) & 1));
  } else if (warp == 2) {
    // ---- activation producer: walks the same ring positions as the ring producer.  For a GEMM unit it waits
    // for the GEMM's input (once per GEMM), then adds the unit's activation tile to the slot (the slot's
    // second arrival); for a KV slot it only arrives.  Whole warp, lane 0 issues.
    int st = 0;
    uint32_t ph = 0;
    long long issued = 0;
    bool ok = true;
    const int kvs = kv_slots(p, c);
    auto advance = [&]() {
      ++issued;
      if (++st == p.w_stages) {
        st = 0;
        ph ^= 1u;
      }
    };
    for (int layer = 0; ok && layer < p.L; ++layer) {
      const long long layer_first = issued;
      for (int g = 0; ok && g < 4; ++g) {
        const Gemm m = gemm_of(p, g);
        const int u0 = unit_begin(m, c), u1 = unit_begin(m, c + 1);
        if (u0 < u1) {
          const unsigned* wc = nullptr;
          unsigned target = static_cast<unsigned>(p.G);
          if (g == 0 && layer > 0) wc = ctr(p, layer - 1, kNorm2);
          if (g == 1) wc = ctr(p, layer, kAtt);
          if (g == 2) wc = ctr(p, layer, kNorm1);
          if (g == 3) {
            wc = ctr(p, layer, kGuf);
            target = static_cast<unsigned>(gemm_of(p, 2).T);
          }
          bool ready = true;
          if (wc && lane == 0) ready = DS_TIMED(p, kStActCtr, cwait(p, wc, target, kErrTimeoutFlag));
          if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          const CUtensorMap* map = p.amaps + g;
          int kb = u0 % m.KB;
          for (int u = u0; u < u1; ++u, kb = (kb + 1 == m.KB) ? 0 : kb + 1) {
            if (!DS_TIMED(p, kStActEmpty, mwait_warp(&s.wempty[st], ph ^ 1u, p, kErrTimeoutProducer))) {
              ok = false;
              break;
            }
            if (lane == 0) {
              evlog(p, layer, 0, static_cast<int>(issued - layer_first));
              mbar_arrive_expect_tx(&s.wfull[st], abytes);
              tma_load_2d(s.wbuf + st * SB + kSlot, map, &s.wfull[st], kb * kBK, 0);
            }
            __syncwarp();
            advance();
          }
        }
        if (g == 0) {
          for (int i = 0; ok && i < kvs; ++i) {  // KV slots carry no activation: plain second arrival
            if (!mwait_warp(&s.wempty[st], ph ^ 1u, p, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            if (lane == 0) mbar_arrive(&s.wfull[st]);
            __syncwarp();
            advance();
          }
        }
      }
    }
    // this warp's activation copies have landed before the CTA can exit
    for (long long i = issued - 1; i >= 0 && i >= issued - p.w_stages; --i)
      mwait_drain(&s.wfull[i % p.w_stages], static_cast<uint32_t>((i / p.w_stages) & 1));
  } else if (warp == 1) {
    // ---- MMA issuer (steps over the ring slots of the KV chunks, which the attention warps consume); the
    // whole warp walks the loop, lane 0 issues
    const uint32_t idesc = idesc_bf16_f32(128, p.BP, false, false);
    const uint32_t wb = smem_u32(s.wbuf);
    const int kvs = kv_slots(p, c);
    int wst = 0;
    uint32_t wph = 0;
    int lt = 0;
    bool ok = true;
    for (int layer = 0; ok && layer < p.L; ++layer) {
      int kcount = 0;
      for (int g = 0; ok && g < 4; ++g) {
        const Gemm m = gemm_of(p, g);
        const int ubeg = unit_begin(m, c), u1 = unit_begin(m, c + 1);
        int u = ubeg, kbs = ubeg % m.KB;  // a segment's first k-block: kbs, then 0 for every later tile
        while (ok && u < u1) {
          const int kb0 = kbs;
          const int kb1 = min(m.KB, kb0 + (u1 - u));
          const bool first_seg = u == ubeg;
          u += kb1 - kb0;
          kbs = 0;
          const int acc = lt & 1;
          const uint32_t use = static_cast<uint32_t>(lt >> 1);
          ++lt;
          if (!DS_TIMED(p, kStMmaT, mwait_warp(&s.tempty[acc], (use & 1u) ^ 1u, p, kErrTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(acc * p.NA * p.BP);
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!DS_TIMED(p, kStMmaW, mwait_warp(&s.wfull[wst], wph, p, kErrTimeoutMma))) {
              ok = false;
              break;
            }
            if (lane == 0) {
              evlog(p, layer, 2, kcount);
              if (first_seg && kb == kb0) trace(p, layer, kTrMmaQkv + g);
              tc_fence_after();
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                // chain k % NA: consecutive MMAs target different accumulators, so they pipeline
                const uint64_t ad = sdesc_sw128(wb + wst * SB + k * 32, 16, 1024);
                const uint64_t bd = sdesc_sw128(wb + wst * SB + kSlot + k * 32, 16, 1024);
                const int q = k % p.NA;
                umma_f16(d + static_cast<uint32_t>(q * p.BP), ad, bd, idesc, (kb != kb0 || k >= p.NA) ? 1u : 0u);
              }
              umma_commit(&s.wempty[wst]);  // frees the weight tile and the activation tile together
            }
            __syncwarp();
            ++kcount;
            if (++wst == p.w_stages) {
              wst = 0;
              wph ^= 1u;
            }
          }
          if (!ok) break;
          if (lane == 0) umma_commit(&s.tfull[acc]);
          __syncwarp();
        }
        if (g == 0) {  // step over this layer's KV slots
          wst += kvs % p.w_stages;
          wph ^= static_cast<uint32_t>((kvs / p.w_stages) & 1);
          if (wst >= p.w_stages) {
            wst -= p.w_stages;
            wph ^= 1u;
          }
          // A parity wait cannot tell a phase from the one two uses later, so before waiting on the o tiles'
          // slots, whose previous phase may be a KV chunk the attention warps have not seen yet, wait until
          // the attention warps are done with every KV slot of the layer.
          if (!DS_TIMED(p, kStMmaA, mwait_warp(s.kvdone, static_cast<uint32_t>(layer & 1), p, kErrTimeoutMma))) ok = false;
        }
      }
    }
    (void)ok;
    // every MMA this warp issued has completed before TMEM is released
    if (lane == 0) umma_commit(s.drain);
    __syncwarp();
    mwait_drain(s.drain, 0);
  } else if (warp >= 4) {
    // ---- compute warps
    int lt = 0;
    const bool epi = warp < 8;
    const bool tr = threadIdx.x == 128;
    // ring position of a layer's first KV slot: this CTA's ring entries per layer times the layer, plus
    // its qkv tiles
    const Gemm mq = gemm_of(p, 0), mo = gemm_of(p, 1), mg = gemm_of(p, 2), md = gemm_of(p, 3);
    const int nq_units = unit_begin(mq, c + 1) - unit_begin(mq, c);
    const int per_layer = nq_units + kv_slots(p, c) + (unit_begin(mo, c + 1) - unit_begin(mo, c)) +
                                (unit_begin(mg, c + 1) - unit_begin(mg, c)) + (unit_begin(md, c + 1) - unit_begin(md, c));
    for (int layer = 0; layer < p.L; ++layer) {
      if (epi) epilogue_phase(p, s, tmem_base, layer, 0, lt);
      if (tr) trace(p, layer, kTrQkvEpi);
      group_wait(p, s, ctr(p, layer, kQkv), static_cast<unsigned>(p.G), kErrTimeoutFlag);
      if (tr) trace(p, layer, kTrQkvWait);
      {
        const long long t0 = clock64();
        attention_phase<REP>(p, s, layer, layer * per_layer + nq_units);
        if (tr) stat_add(p, kStAttention, clock64() - t0);
      }
      if (threadIdx.x == 128) mbar_arrive(s.kvdone);  // after the item loop's last compute barrier
      group_arrive(p, ctr(p, layer, kAtt));
      if (tr) trace(p, layer, kTrAtt);
      if (epi) epilogue_phase(p, s, tmem_base, layer, 1, lt);
      if (tr) trace(p, layer, kTrOEpi);
      group_wait(p, s, ctr(p, layer, kO), static_cast<unsigned>(p.G), kErrTimeoutFlag);
      if (tr) trace(p, layer, kTrOWait);
      {
        const long long t0 = clock64();
        norm_phase(p, s, layer, false);
        if (tr) stat_add(p, kStNorm, clock64() - t0);
      }
      group_arrive(p, ctr(p, layer, kNorm1));
      if (tr) trace(p, layer, kTrNorm1);
      if (epi) {
        epilogue_phase(p, s, tmem_base, layer, 2, lt);
        if (tr) trace(p, layer, kTrGuEpi);
        epilogue_phase(p, s, tmem_base, layer, 3, lt);
        if (tr) trace(p, layer, kTrDownEpi);
      }
      group_wait(p, s, ctr(p, layer, kDown), static_cast<unsigned>(p.G), kErrTimeoutFlag);
      if (tr) trace(p, layer, kTrDownWait);
      norm_phase(p, s, layer, true);
      group_arrive(p, ctr(p, layer, kNorm2));
      if (tr) trace(p, layer, kTrNorm2);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) stat_add(p, kStTotal, clock64() - t_start);
  __syncthreads();
  if (p.trace && threadIdx.x < 16)
    p.trace[static_cast<long long>(p.G) * p.L * 16 + blockIdx.x * 16 + threadIdx.x] +=
        static_cast<long long>(ds_stats[threadIdx.x]);
  if (warp == 3) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace ds

// ------------------------------------------------------------------ host
namespace {

struct DsGeom {
  int w_stages, slot_bytes, smem;
};

DsGeom ds_geom(int BP, int rep) {
  constexpr int kBudget = 227 * 1024;
  const int slot = ds::kSlot + ds::a_stage_bytes(BP);  // multiple of 2 KB: every slot stays 1 KB aligned
  const int fixed = 1024 /* alignment */ + ds::merge_floats(rep) * 4 + ds::kMaxItems * (rep + 2) * ds::kD * 2 +
                    16 * 4 + 640 /* barriers, TMEM holder, flags */;
  // a multiple of 4: each attention group's parity waits then find the slot's previous phase among the
  // group's own earlier chunks (decode_step_kernel's attention phase)
  int w_stages = std::min((kBudget - fixed) / slot, 12) & ~3;
  DsGeom g;
  g.w_stages = w_stages;
  g.slot_bytes = slot;
  g.smem = fixed + w_stages * slot;
  return g;
}

}  // namespace

// Tensor maps of the persistent decode step, as CPU uint8 tensors of 128-byte entries (to be copied to the
// device): weights [L*4] (qkv, o, gate/up, down per layer) followed by the [L*2] K / V cache layers
// ([B, Hkv, Tmax, D] each, seen as [B*Hkv*Tmax, D] in 64 x 64 boxes), and activations [4] (xn, o, hn, act).
std::vector<at::Tensor> decode_step_maps(std::vector<at::Tensor> weights, std::vector<at::Tensor> caches,
                                         std::vector<at::Tensor> acts, int64_t BP) {
  TORCH_CHECK(acts.size() == 4, "decode_step_maps: four activation buffers");
  TORCH_CHECK(caches.size() * 2 == weights.size(), "decode_step_maps: a K and a V cache per layer");
  auto opts = at::TensorOptions().dtype(at::kByte);
  at::Tensor wm = at::empty({static_cast<int64_t>(weights.size() + caches.size()), 128}, opts);
  at::Tensor am = at::empty({4, 128}, opts);
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  for (size_t i = 0; i < weights.size(); ++i) {
    const at::Tensor& w = weights[i];
    TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, "decode_step_maps: weight ", i);
    TORCH_CHECK(w.size(0) % ds::kTileN == 0 && w.size(1) % ds::kBK == 0, "decode_step_maps: weight shape");
    const CUtensorMap m = make_tmap_2d_bf16(w.data_ptr(), w.size(1), w.size(0), w.size(1), ds::kBK, ds::kTileN);
    std::memcpy(wm.data_ptr<uint8_t>() + i * 128, &m, 128);
  }
  for (size_t i = 0; i < caches.size(); ++i) {
    const at::Tensor& kv = caches[i];
    TORCH_CHECK(kv.dim() == 4 && kv.is_contiguous() && kv.scalar_type() == at::kBFloat16 && kv.size(3) == ds::kD,
                "decode_step_maps: cache layer [B, Hkv, Tmax, 128]");
    const int64_t rows = kv.size(0) * kv.size(1) * kv.size(2);
    const CUtensorMap m = make_tmap_2d_bf16(kv.data_ptr(), ds::kD, rows, ds::kD, 64, ds::kKC);
    std::memcpy(wm.data_ptr<uint8_t>() + (weights.size() + i) * 128, &m, 128);
  }
  for (int i = 0; i < 4; ++i) {
    const at::Tensor& a = acts[i];
    TORCH_CHECK(a.dim() == 2 && a.is_contiguous() && a.scalar_type() == at::kBFloat16, "decode_step_maps: activation");
    const CUtensorMap m = make_tmap_2d_bf16(a.data_ptr(), a.size(1), a.size(0), a.size(1), ds::kBK, static_cast<int>(BP));
    std::memcpy(am.data_ptr<uint8_t>() + i * 128, &m, 128);
  }
  return {wm, am};
}

// Sync words the launch needs (zeroed by decode_step before the kernel).
int64_t decode_step_sync_words(int64_t L, int64_t F, int64_t B) {
  (void)B;
  return (1 + L * ds::kCtrPerLayer) * ds::kLine + L * (2 * F / ds::kTileN);
}

// dims = {L, B, H, nq, nkv, F, Tmax}
void decode_step(at::Tensor wmaps, at::Tensor amaps, at::Tensor layers, at::Tensor x, at::Tensor h1, at::Tensor xn,
                 at::Tensor o, at::Tensor hn, at::Tensor act, at::Tensor ws, at::Tensor ssq, at::Tensor sync,
                 at::Tensor lens, at::Tensor delta, at::Tensor inv_freq, c10::optional<at::Tensor> lead,
                 c10::optional<at::Tensor> share_len, std::vector<int64_t> dims, double eps, double scale,
                 c10::optional<at::Tensor> trace) {
  TORCH_CHECK(dims.size() == 7, "decode_step: dims = {L, B, H, nq, nkv, F, Tmax}");
  const c10::cuda::CUDAGuard guard(x.device());
  ds::Params p{};
  p.L = static_cast<int>(dims[0]);
  p.B = static_cast<int>(dims[1]);
  p.H = static_cast<int>(dims[2]);
  p.nq = static_cast<int>(dims[3]);
  p.nkv = static_cast<int>(dims[4]);
  p.F = static_cast<int>(dims[5]);
  p.Tmax = static_cast<int>(dims[6]);
  p.BP = std::max(16, (p.B + 15) / 16 * 16);
  p.NA = p.BP <= 64 ? 4 : 2;
  const int rep = p.nq / p.nkv;
  TORCH_CHECK(p.B >= 1 && p.BP <= 128, "decode_step: batch must be 1..128");
  TORCH_CHECK(p.nq % p.nkv == 0 && (rep == 1 || rep == 2 || rep == 4 || rep == 8), "decode_step: GQA ratio");
  TORCH_CHECK(p.B * p.nkv <= ds::kMaxItems * num_sms(x.device().index()), "decode_step: too many attention items");
  TORCH_CHECK(p.B * (p.H / ds::kTileN) <= 4 * 8 * num_sms(x.device().index()), "decode_step: too many norm items");
  TORCH_CHECK(p.H % ds::kTileN == 0 && p.H <= 4096 && (2 * p.F) % ds::kTileN == 0 && p.F % ds::kBK == 0,
              "decode_step: hidden / intermediate sizes");
  TORCH_CHECK(sync.numel() >= decode_step_sync_words(p.L, p.F, p.B) && sync.scalar_type() == at::kInt,
              "decode_step: sync words");
  TORCH_CHECK(ssq.numel() >= 2 * p.B * (p.H / ds::kTileN) && ssq.scalar_type() == at::kFloat, "decode_step: ssq");
  TORCH_CHECK(wmaps.numel() >= static_cast<int64_t>(p.L) * 6 * 128 && amaps.numel() >= 4 * 128, "decode_step: maps");
  TORCH_CHECK(lens.scalar_type() == at::kInt && delta.scalar_type() == at::kLong, "decode_step: int32 lengths, int64 deltas");
  const int dev = x.device().index();
  p.G = num_sms(dev);
  const DsGeom geo = ds_geom(p.BP, rep);
  p.w_stages = geo.w_stages;
  p.slot_bytes = geo.slot_bytes;
  TORCH_CHECK(p.w_stages >= 4, "decode_step: shared memory too small");
  p.eps = static_cast<float>(eps);
  p.scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  p.wmaps = reinterpret_cast<const CUtensorMap*>(wmaps.data_ptr());
  p.amaps = reinterpret_cast<const CUtensorMap*>(amaps.data_ptr());
  p.layers = reinterpret_cast<const ds::Layer*>(layers.data_ptr());
  auto bp = [](at::Tensor& t) { return reinterpret_cast<bf16*>(t.data_ptr()); };
  p.x = bp(x);
  p.h1 = bp(h1);
  p.xn = bp(xn);
  p.o = bp(o);
  p.hn = bp(hn);
  p.act = bp(act);
  p.ws = ws.data_ptr<float>();
  p.ssq = ssq.data_ptr<float>();
  p.lens = lens.data_ptr<int>();
  p.delta = delta.data_ptr<int64_t>();
  p.inv_freq = inv_freq.data_ptr<float>();
  const bool share = lead.has_value() && lead->defined() && share_len.has_value() && share_len->defined();
  p.lead = share ? lead->data_ptr<int>() : nullptr;
  p.share_len = share ? share_len->data_ptr<int>() : nullptr;
  p.sync = reinterpret_cast<unsigned*>(sync.data_ptr<int>());
  p.err = err_word(dev);
  p.trace = (trace.has_value() && trace->defined()) ? reinterpret_cast<long long*>(trace->data_ptr<int64_t>()) : nullptr;
  if (p.trace) TORCH_CHECK(trace->numel() >= static_cast<int64_t>(p.G) * (p.L + 1) * 16 + 3 * 256, "decode_step: trace size");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  VLM_CUDA_CHECK(cudaMemsetAsync(sync.data_ptr(), 0, sizeof(int) * decode_step_sync_words(p.L, p.F, p.B), st));
  auto launch = [&](auto kern) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, geo.smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.G);
    cfg.blockDim = dim3(ds::kThreads);
    cfg.dynamicSmemBytes = geo.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phases wait on one another
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VLM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p));
    note_launch();
  };
  if (rep == 4)
    launch(ds::decode_step_kernel<4>);
  else if (rep == 2)
    launch(ds::decode_step_kernel<2>);
  else if (rep == 8)
    launch(ds::decode_step_kernel<8>);
  else
    launch(ds::decode_step_kernel<1>);
}

// Partial-slot capacity (floats) the launch needs for batch B: max over the four GEMMs of slots x B x N.
int64_t decode_step_ws_floats(std::vector<int64_t> dims, int64_t grid) {
  const int64_t B = dims[1], H = dims[2], nq = dims[3], nkv = dims[4], F = dims[5];
  const int64_t Ns[4] = {(nq + 2 * nkv) * ds::kD, H, 2 * F, H};
  const int64_t Ks[4] = {H, nq * ds::kD, H, F};
  int64_t best = 0;
  for (int g = 0; g < 4; ++g) {
    const int64_t T = Ns[g] / ds::kTileN, KB = Ks[g] / ds::kBK, U = T * KB;
    const int64_t Gg = std::min(grid, U);
    auto cta = [&](int64_t u) { return ((u + 1) * Gg - 1) / U; };
    int64_t mx = 1;
    for (int64_t t = 0; t < T; ++t) mx = std::max(mx, cta(t * KB + KB - 1) - cta(t * KB) + 1);
    best = std::max(best, mx * B * Ns[g]);
  }
  return best;
}

}  // namespace vlm
