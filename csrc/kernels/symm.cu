// Symmetric peer memory for the fused tensor-parallel reductions: one
// cudaMalloc'd buffer per rank, exported with a CUDA IPC handle and opened in
// every peer process of the node (NVLink / NVSwitch peer mappings), plus a
// one-GPU self-test of the push/reduce protocol (world = 1, loopback).
#include <cuda_runtime.h>
#include <cstring>
#include "symm.cuh"
#include "torch_glue.h"
#include <ATen/ops/empty.h>
#include <ATen/ops/from_blob.h>

using namespace moet;

#define SYMM_CHECK(x)                                                                        \
  do {                                                                                       \
    cudaError_t e_ = (x);                                                                    \
    TORCH_CHECK(e_ == cudaSuccess, #x " failed: ", cudaGetErrorString(e_));                  \
  } while (0)

// -> (device pointer, 64-byte IPC handle as a CPU uint8 tensor); memory zeroed.
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t bytes) {
  TORCH_CHECK(bytes > 0, "symm_alloc: size");
  void* p = nullptr;
  SYMM_CHECK(cudaMalloc(&p, (size_t)bytes));
  SYMM_CHECK(cudaMemset(p, 0, (size_t)bytes));
  SYMM_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  SYMM_CHECK(cudaIpcGetMemHandle(&h, p));
  at::Tensor t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), t};
}

int64_t symm_open(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.device().is_cpu(), "symm_open: handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  SYMM_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { SYMM_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }
void symm_free(int64_t ptr) { SYMM_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

// A uint8 CUDA tensor aliasing [ptr, ptr + bytes) (no ownership).
at::Tensor symm_view(int64_t ptr, int64_t bytes, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), {bytes},
                       at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (int)device));
}

namespace {
// Loopback / protocol test: every CTA pushes x[rows, n] (f32) as its partial,
// then a second kernel reduces into out = resid + sum of partials.
__global__ void ar_push_test_kernel(ArDesc d, const float* __restrict__ x, int n) {
  const unsigned long long epoch = ar_epoch(d);
  const int row = blockIdx.x;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[(size_t)row * n + i];
    for (int p = 0; p < d.world; p++) ar_slot(d, p, epoch, d.rank)[(size_t)row * n + i] = v;
  }
  ar_producer_arrive(d, epoch);
}

__global__ void ar_reduce_test_kernel(ArDesc d, const float* __restrict__ resid, float* __restrict__ out, int n) {
  const unsigned long long epoch = ar_epoch(d);
  const int row = blockIdx.x;
  const bool ok = ar_consumer_wait(d, epoch);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float s = resid ? resid[(size_t)row * n + i] : 0.f;
    if (ok)
      for (int r = 0; r < d.world; r++) s += ar_slot(d, d.rank, epoch, r)[(size_t)row * n + i];
    out[(size_t)row * n + i] = s;
  }
  ar_consumer_done(d);
}
}  // namespace

// push_only / reduce_only split the two halves so tests can leave a flag unset
// (the reduce then times out with kTimeout instead of hanging).
void ar_test(at::Tensor desc, at::Tensor x, c10::optional<at::Tensor> resid, at::Tensor out, int64_t mode) {
  ArDesc d = ar_desc_from(desc);
  const int rows = x.size(0), n = x.size(1);
  TORCH_CHECK(x.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat && x.is_contiguous() &&
                  out.is_contiguous() && (int64_t)rows * n <= d.cap, "ar_test: f32 contiguous, rows*n <= cap");
  auto stream = at::cuda::getCurrentCUDAStream();
  if (mode != 2) ar_push_test_kernel<<<rows, 128, 0, stream>>>(d, x.data_ptr<float>(), n);
  if (mode != 1)
    ar_reduce_test_kernel<<<rows, 128, 0, stream>>>(d, (const float*)opt_ptr(resid), out.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
