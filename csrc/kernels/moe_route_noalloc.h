// Pair-list builder that allocates nothing (C ABI).
//
// This entry point has no counterpart in the reference.  It exists for
// callers that cannot call cudaMalloc: code embedded in a host runtime
// without PyTorch's caching allocator (plain C/C++ schedulers, other
// language bindings), and serving processes that have already handed all
// free HBM to the KV cache and expert pools, where a late cudaMalloc could
// fail or fragment memory.  The caller passes inputs and outputs; the
// per-routing scratch the kernel needs is a fixed array compiled into the
// library (see MOET_NOALLOC_MAX_ROUTINGS).
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest num_tokens * top_k one call accepts (8192 tokens x top-8).  The
// scratch array holds one int per routing: 256 KiB, kept on every GPU that
// loads the library until the process exits.
#define MOET_NOALLOC_MAX_ROUTINGS 65536

// Return codes (besides these, a positive value is a cudaError_t).
#define MOET_NOALLOC_OK 0
#define MOET_NOALLOC_EINVAL (-1)   // bad argument (null pointer, k/E/rows out of range, max_pairs too
                                   // small, pairs not 16-byte aligned)
#define MOET_NOALLOC_ETOOBIG (-2)  // num_tokens * top_k exceeds MOET_NOALLOC_MAX_ROUTINGS

// Groups the num_tokens*top_k routings in topk_ids [num_tokens, top_k]
// (int32 expert ids) by expert and cuts each expert's rows into pairs of at
// most rows_per_pair rows.  Outputs (device pointers, caller-owned):
//   sorted_tok [R]        token of each expert-sorted row
//   pos_of     [R]        routing t*top_k+j -> sorted row
//   pairs      [max_pairs][4] {expert, first sorted row, n rows, 0};
//                          max_pairs >= R/rows_per_pair + min(num_experts, R);
//                          16-byte aligned (each record is one 16-byte store)
//   n_pairs    [1]        number of pairs written
//   status     [1]        caller-zeroed: the kernel only ever sets it (to 1
//                          when an expert id is out of range; such a routing
//                          is counted under expert 0) and never clears it
// Enqueued on `stream`; returns before the kernel finishes.
//
// Set-up: the first call on each device (with that device current) looks up
// the device address of the scratch array; make that first call before any
// stream capture on the device.  All calls share the one array and it keeps
// whatever the last call left in it (every slot a call reads it writes
// first, so nothing needs clearing); calls that overlap on the GPU -- on
// different streams, or from different host threads -- race on it and must
// be serialised by the caller.
int moet_build_pairs_noalloc(const int* topk_ids, int num_tokens, int top_k, int num_experts,
                             int rows_per_pair, int* sorted_tok, int* pos_of, int* pairs, int max_pairs,
                             int* n_pairs, int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
