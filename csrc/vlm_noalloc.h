// C interface of the allocation-free decode attention entry point (defined in attention.cu).
//
// Declaration: this interface has no counterpart in the reference project.  It serves callers that
// cannot allocate device memory at call time: an inference host whose pool allocator owns all device
// memory (an allocation behind its back breaks its accounting and can fail under its memory cap), a
// latency-critical loop where an allocation would be a synchronising driver call, or plugin code that
// may only touch the buffers it was handed.  The caller passes inputs and outputs; the key-split
// partial results live in a fixed 4 MiB device array of the library and timed-out waits are recorded
// in a fixed device status word, both resolved once per device by the first call on it (make that
// first call before any CUDA-graph capture).  Calls on one device share the array, so calls that
// overlap on the GPU race and must be serialised by the caller.  Neither function allocates device
// memory or lets a C++ exception escape.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// q [B, Hq, D] bf16, k_cache / v_cache [B, Hkv, Tmax, D] bf16, lengths [B] int32 (valid keys per
// sequence), out [B, Hq, D] bf16: device pointers to contiguous buffers.  stream: a cudaStream_t
// (0 = legacy default stream).  Computes out = softmax(q . K^T * scale) . V over the first lengths[b]
// keys of each sequence, Hq / Hkv query heads per key head.  Supported (D, Hq / Hkv): (128, 1|2|4),
// (64, 4), (32, 2).  Needs B * Hq * splits * (D + 2) <= 2^20 floats of scratch, where splits >= 2 is
// the number of key splits the launch picks.
// Returns 0 ok, -1 unsupported shape, -2 problem exceeds the scratch array, -3 CUDA error.
int vlmrl_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* lengths,
                                   void* out, int B, int Hq, int Hkv, int Tmax, int D, float scale, void* stream);

// Waits for `stream`, stores the current device's status word in *status (0 = no bounded wait ran
// out since the last read, else the first error code recorded, after which the output of that call
// is undefined) and clears it.  Returns 0, or -3 on a CUDA error.
int vlmrl_decode_attention_noalloc_status(void* stream, int* status);

#ifdef __cplusplus
}
#endif
