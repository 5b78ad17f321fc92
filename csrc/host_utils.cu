// Host helpers: tensor-map encoding through the driver entry point (no libcuda link),
// cached device properties and the per-device error word.
#include <ATen/cuda/CUDAContext.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "host_utils.h"

namespace vlm {

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    VLM_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

std::mutex g_mu;
std::atomic<int64_t> g_launches{0};
std::vector<int*> g_err(64, nullptr);
std::vector<int> g_sms(64, 0);
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(); }

int* err_word(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err[device]) {
    int* p = nullptr;
    VLM_CUDA_CHECK(cudaMalloc(&p, sizeof(int) * 4));
    VLM_CUDA_CHECK(cudaMemset(p, 0, sizeof(int) * 4));
    g_err[device] = p;
  }
  return g_err[device];
}

unsigned* grid_barrier_words(int device) {
  static std::vector<unsigned*> words(64, nullptr);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!words[device]) {
    unsigned* p = nullptr;
    VLM_CUDA_CHECK(cudaMalloc(&p, sizeof(unsigned) * 4));
    VLM_CUDA_CHECK(cudaMemset(p, 0, sizeof(unsigned) * 4));
    words[device] = p;
  }
  return words[device];
}

int64_t read_and_clear_error(int64_t device) {
  int* w = err_word(static_cast<int>(device));
  int h = 0;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  VLM_CUDA_CHECK(cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, st));
  VLM_CUDA_CHECK(cudaStreamSynchronize(st));
  if (h) VLM_CUDA_CHECK(cudaMemsetAsync(w, 0, sizeof(int), st));
  return h;
}

std::vector<int64_t> read_error_words(int64_t device) {
  int* w = err_word(static_cast<int>(device));
  int h[4] = {0, 0, 0, 0};
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  VLM_CUDA_CHECK(cudaMemcpyAsync(h, w, sizeof(h), cudaMemcpyDeviceToHost, st));
  VLM_CUDA_CHECK(cudaStreamSynchronize(st));
  if (h[0] || h[1] || h[2] || h[3]) VLM_CUDA_CHECK(cudaMemsetAsync(w, 0, sizeof(h), st));
  return {h[0], h[1], h[2], h[3]};
}

int num_sms(int device) {
  if (!g_sms[device]) {
    int v = 0;
    VLM_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
    g_sms[device] = v;
  }
  return g_sms[device];
}

CUtensorMap make_tmap_2d_bf16(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "tensor map base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0 || outer == 1, "tensor map row stride must be a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r), " (inner=", inner,
              ", outer=", outer, ", ld=", ld, ", box=", box_inner, "x", box_outer, ")");
  return m;
}

}  // namespace vlm
