// Allocation-free variant of the tcgen05 gated-attention backward.
//
// This entry point has no counterpart in the reference framework. It is for
// callers that cannot allocate device memory (allocator or pool callbacks,
// hosts that reserve all memory at start-up, runtimes that forbid
// cudaMalloc once work is running). Its scratch is a fixed file-scope device
// array; see the implementation in gated_tc_bwd.cu for the size limits and
// the rule that calls overlapping on the GPU race on that array.
//
// Inputs are the tensors of the forward pass (bf16 q/k/v/out/grad laid out
// [batch, rows, heads, head_dim], int32 positions [batch, queries], fp32
// rc [batch, queries, heads, head_dim] and pr/zr/lse [batch, queries, heads]);
// dq/dk/dv are bf16 outputs of the same layouts as q/k/v. head_dim is 64 or
// 128, block 16/32/64/128. The first call on a device looks up the device
// address of the scratch array for that device (the device current at the
// call); make that first call before any stream capture. Returns 0 on success;
// otherwise writes a message into error_message (if error_capacity > 0). A
// return of 0 means the kernels were enqueued; whether they finished their
// bounded waits is known only after the stream is synchronised, from
// eb_gated_attention_bwd_noalloc_status (site != 0: the gradients of that call
// are incomplete).
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

int eb_gated_attention_bwd_noalloc(const void* grad, const void* q, const void* k, const void* v, const int* pos,
                                   const void* out, const float* rc, const float* pr, const float* zr,
                                   const float* lse, void* dq, void* dk, void* dv, int batch, int queries, int keys,
                                   int heads, int head_dim, int block, void* stream, char* error_message,
                                   int error_capacity);

// Reads and clears the bounded-wait record of the calls above on `device`
// (*site = 0: no wait gave up; otherwise the wait's site id and *cta the CTA).
// Call after synchronising. Uses cudaMemcpy/cudaMemset, allocates nothing.
int eb_gated_attention_bwd_noalloc_status(int device, int* site, int* cta, char* error_message, int error_capacity);

#ifdef __cplusplus
}
#endif
