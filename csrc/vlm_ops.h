// Declarations shared between kernel translation units and the Python bindings.
#pragma once

#include <torch/extension.h>

#include <tuple>
#include <vector>

namespace vlm {

struct SkMeta;
struct DecFuse;

struct VocabArgs {
  const int64_t* targets;
  const float* lse;
  const float* ent;
  const float* g_lp;
  const float* g_ent;
  float* part;
  int* cand_i = nullptr;  // EPI_TOPK: per (row, tile) top-k indices (values go to part)
  int topk = 0;
};

// Fused all-gather of a GEMM's weight operand: B is a view into the local copy of a flat parameter unit
// (starting at dst_base) whose equal shards of shard_bytes live at srcs[r] (peer mappings for r != rank).
struct GatherArgs {
  std::vector<int64_t> srcs;
  int64_t dst_base;
  int64_t shard_bytes;
  at::Tensor flags;  // int32 [>= chunks], zero
  at::Tensor ctr;    // int32 [2], zero
};

// gemm_sm100.cu
void gemm(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux, bool a_kmajor,
          bool b_kmajor, double alpha, int64_t epi, bool accumulate);
void gemm_ex(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux,
             bool a_kmajor, bool b_kmajor, double alpha, int64_t epi, bool accumulate, const VocabArgs* vocab,
             int force_bn, at::Tensor* partials_out, SkMeta* meta_out, const GatherArgs* gather = nullptr,
             const DecFuse* fuse = nullptr);
// Decode GEMMs (x [B, K] . w^T) whose consumer runs inside the GEMM after a grid-wide barrier: the same
// results as gemm_partials followed by dec_qkv / dec_residual_norm / dec_swiglu, one launch each.
at::Tensor dec_gemm_qkv(at::Tensor x, at::Tensor w, at::Tensor bias, at::Tensor qw, at::Tensor kw, at::Tensor lengths,
                        at::Tensor delta, at::Tensor inv_freq, at::Tensor kc, at::Tensor vc, int64_t nq, int64_t nkv,
                        double eps);
std::tuple<at::Tensor, at::Tensor> dec_gemm_residual_norm(at::Tensor x, at::Tensor w, at::Tensor residual, at::Tensor nw,
                                                          double eps);
at::Tensor dec_gemm_swiglu(at::Tensor x, at::Tensor w);
// gemm() whose B rows are all-gathered from the ranks' shards inside the kernel (see GatherArgs)
void gemm_gather(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux,
                 bool a_kmajor, bool b_kmajor, double alpha, int64_t epi, bool accumulate, std::vector<int64_t> srcs,
                 int64_t dst_base, int64_t shard_bytes, at::Tensor flags, at::Tensor ctr);
// Copy byte ranges [starts[i], ends[i]) of a flat unit from the ranks' shards into the local copy (the small
// leaves a fused gather GEMM does not cover).
void unit_gather(std::vector<int64_t> srcs, int64_t dst_base, int64_t shard_bytes, std::vector<int64_t> starts,
                 std::vector<int64_t> ends);
// Stream-K partial sums of A.B^T without an epilogue: (ws [slots, M, N] fp32, meta) for the fused consumers.
std::tuple<at::Tensor, std::vector<int64_t>> gemm_partials(at::Tensor A, at::Tensor B);
std::tuple<at::Tensor, std::vector<int64_t>> gemm_partials_traced(at::Tensor A, at::Tensor B, at::Tensor trace);
// decode_gemm.cu: skinny (M <= 64) partial sums in the stream-K layout; static_weights lets the first weight
// chunks go out before the wait on the previous kernel.
bool skinny_enabled();
std::tuple<at::Tensor, std::vector<int64_t>> skinny_partials(const at::Tensor& x, const at::Tensor& w,
                                                             bool static_weights);
// While on, GEMMs prefetch their K-major B operand before waiting on the previous kernel (PDL).
void set_static_weights(bool on);

// decode.cu: consumers of stream-K partials fused with the decode step's memory-bound ops
at::Tensor dec_qkv(at::Tensor ws, std::vector<int64_t> meta, at::Tensor bias, at::Tensor qw, at::Tensor kw,
                   at::Tensor lengths, at::Tensor delta, at::Tensor inv_freq, at::Tensor kc, at::Tensor vc, int64_t nq,
                   int64_t nkv, double eps,
                   c10::optional<at::Tensor> prefetch = c10::nullopt,
                   c10::optional<at::Tensor> block_table = c10::nullopt);
std::tuple<at::Tensor, at::Tensor> dec_residual_norm(at::Tensor ws, std::vector<int64_t> meta, at::Tensor residual,
                                                     at::Tensor w, double eps,
                                                     c10::optional<at::Tensor> prefetch = c10::nullopt);
at::Tensor dec_swiglu(at::Tensor ws, std::vector<int64_t> meta, c10::optional<at::Tensor> prefetch = c10::nullopt);

// elementwise.cu
void rms_norm_fwd(at::Tensor x, at::Tensor w, at::Tensor y, at::Tensor rstd, double eps);
void rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor dx, at::Tensor dw,
                  at::Tensor add);
void layer_norm_fwd(at::Tensor x, at::Tensor w, at::Tensor b, at::Tensor y, double eps);
void qk_norm_rope_fwd(at::Tensor qkv, at::Tensor qw, at::Tensor kw, at::Tensor pos, at::Tensor inv_freq, at::Tensor ax,
                      at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor rq, at::Tensor rk, int64_t nq, int64_t nkv,
                      double eps);
void qk_norm_rope_bwd(at::Tensor dq, at::Tensor dk, at::Tensor dv, at::Tensor qkv, at::Tensor qw, at::Tensor kw,
                      at::Tensor pos, at::Tensor inv_freq, at::Tensor ax, at::Tensor rq, at::Tensor rk, at::Tensor dqkv,
                      at::Tensor dqw, at::Tensor dkw, int64_t nq, int64_t nkv, double eps);
void vision_rope(at::Tensor qkv, at::Tensor rc, at::Tensor q, at::Tensor k, at::Tensor v, int64_t n_heads,
                 int64_t style);
void swiglu_bwd(at::Tensor d_act, at::Tensor pre, at::Tensor out);
void embed(at::Tensor tokens, at::Tensor table, at::Tensor out);
void scatter_rows(at::Tensor h, at::Tensor rows, at::Tensor src, bool add);
void embed_bwd(at::Tensor tokens, at::Tensor dh, at::Tensor dtable);
void kv_write(at::Tensor k, at::Tensor v, at::Tensor kc, at::Tensor vc, at::Tensor seq, at::Tensor pos,
              c10::optional<at::Tensor> block_table);
void adamw(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor ph, at::Tensor scale, double lr, double b1,
           double b2, double eps, double wd, int64_t step);
void sq_norm_acc(at::Tensor x, at::Tensor out);
void patchify(at::Tensor images, at::Tensor ms, at::Tensor out, int64_t patch, int64_t temporal, int64_t merge);

// attention.cu
void flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu, at::Tensor o, at::Tensor lse,
                    int64_t max_seqlen, bool causal, double scale, c10::optional<at::Tensor> pre);
void flash_attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                    at::Tensor cu, at::Tensor dq, at::Tensor dk, at::Tensor dv, int64_t max_seqlen, bool causal,
                    double scale, c10::optional<at::Tensor> pre, c10::optional<at::Tensor> xq);
// lead / share_len (int32 [B], optional): keys [0, share_len[b]) of row b may be read from row lead[b].
// block_table (int32 [B, blocks], optional): kc / vc are block pools [NB, Hkv, 64, D] (kv_layout.cuh).
void decode_attn(at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor lens, at::Tensor o, double scale,
                 c10::optional<at::Tensor> prefetch = c10::nullopt, c10::optional<at::Tensor> lead = c10::nullopt,
                 c10::optional<at::Tensor> share_len = c10::nullopt,
                 c10::optional<at::Tensor> block_table = c10::nullopt);

// sampler.cu
void sample(at::Tensor logits, at::Tensor tok, at::Tensor lp, at::Tensor step, at::Tensor seed, double temperature,
            int64_t top_k, double top_p, int64_t row_offset);

// vocab.cu
void vocab_logprob_fwd(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor logp, at::Tensor ent, at::Tensor lse);
void vocab_logprob_bwd(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, at::Tensor ent, at::Tensor g_lp,
                       at::Tensor g_ent, at::Tensor dh, at::Tensor dw);

// decode.cu (tensor-parallel decode)
void tp_step_begin(int64_t epoch_ptr, int64_t device);
std::tuple<at::Tensor, at::Tensor> dec_residual_norm_tp(at::Tensor ws, std::vector<int64_t> meta, at::Tensor res,
                                                        at::Tensor w, double eps, std::vector<int64_t> slots,
                                                        int64_t slot_off_bytes, int64_t max_batch, int64_t epoch_ptr,
                                                        int64_t rank);

// symm.cu (peer-memory collectives)
int64_t symm_alloc(int64_t bytes, int64_t device);
void symm_free(int64_t ptr, int64_t device);
at::Tensor symm_ipc_handle(int64_t ptr, int64_t device);
int64_t symm_open(at::Tensor handle, int64_t device);
void symm_close(int64_t ptr, int64_t device);
at::Tensor symm_view(int64_t base, int64_t offset_bytes, std::vector<int64_t> sizes, at::ScalarType dtype,
                     int64_t device);
void rs_pull(std::vector<int64_t> bufs, int64_t unit_off_bytes, int64_t shard_off, at::Tensor out, bool accumulate,
             std::vector<int64_t> sigs, int64_t slot, int64_t epoch, int64_t rank, int64_t max_ctas);
int64_t adamw_push(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, std::vector<int64_t> dst,
                   int64_t dst_off_bytes, at::Tensor scale, double lr, double b1, double b2, double eps, double wd,
                   int64_t step, std::vector<int64_t> sigs, int64_t slot, int64_t rank);
void peer_wait(int64_t local_sig, int64_t slot, int64_t target, int64_t rank, int64_t world, int64_t device,
               int64_t budget_cycles);
void peer_barrier(std::vector<int64_t> sigs, int64_t slot, int64_t epoch, int64_t rank, int64_t device);

// sampler.cu: lm_head fused with the top-k / top-p sampler (logits never materialised)
void lm_head_sample(at::Tensor h, at::Tensor w, at::Tensor tok, at::Tensor lp, at::Tensor step, at::Tensor seed,
                    double temperature, int64_t top_k, double top_p, int64_t row_offset);
// Vocab-parallel lm_head + sampler for tensor-parallel decode: w is this rank's [V_shard, H] rows starting at
// vocab_offset; the shards' top-k survivors are exchanged through the IPC-shared `slots` buffers (tagged by
// the decode step counter at epoch_ptr) and every rank draws the same token.
void lm_head_sample_tp(at::Tensor h, at::Tensor w, int64_t vocab_offset, at::Tensor tok, at::Tensor lp,
                       at::Tensor step, at::Tensor seed, double temperature, int64_t top_k, double top_p,
                       int64_t row_offset, std::vector<int64_t> slots, int64_t slot_off_bytes, int64_t epoch_ptr,
                       int64_t rank);

// decode_step.cu (persistent decode step)
std::vector<at::Tensor> decode_step_maps(std::vector<at::Tensor> weights, std::vector<at::Tensor> caches,
                                         std::vector<at::Tensor> acts, int64_t BP);
int64_t decode_step_sync_words(int64_t L, int64_t F, int64_t B);
int64_t decode_step_ws_floats(std::vector<int64_t> dims, int64_t grid);
void decode_step(at::Tensor wmaps, at::Tensor amaps, at::Tensor layers, at::Tensor x, at::Tensor h1, at::Tensor xn,
                 at::Tensor o, at::Tensor hn, at::Tensor act, at::Tensor ws, at::Tensor ssq, at::Tensor sync,
                 at::Tensor lens, at::Tensor delta, at::Tensor inv_freq, c10::optional<at::Tensor> lead,
                 c10::optional<at::Tensor> share_len, std::vector<int64_t> dims, double eps, double scale,
                 c10::optional<at::Tensor> trace);

// host_utils.cu
int64_t read_and_clear_error(int64_t device);
int64_t launch_count();

}  // namespace vlm
