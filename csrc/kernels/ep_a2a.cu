// Expert-parallel dispatch over peer memory (protocol and buffer layout in ep_a2a.cuh).
// The owner's wait + pair list is ep_recv_pairs (moe_route.cu, beside the pair builder),
// the return leg is fused into the w2 expert GEMV's epilogue and the source's wait into
// moe_combine (moe_w2.cu).
//
// This is the decode-sized counterpart of the all-to-all algorithm in
// vllm_moet_b200/parallel/ep.py (data-parallel attention + expert-parallel MoE); the
// reference serves experts replicated or TP-sharded only (its W2 path refuses EP,
// patch/vllm-moet-v0.24.0.patch:4750-4753).
#include "ep_a2a.cuh"
#include "torch_glue.h"

namespace moet {

// grid = max(T, 1) CTAs.  CTA t copies token t's e4m3 row and scales once per top-k slot
// to the slot's owner (peer stores) and writes the slot's metadata on every rank.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpDesc d, const uint8_t* __restrict__ xq,
                                                          long long xq_stride, const uint8_t* __restrict__ xs,
                                                          long long xs_stride, const int* __restrict__ ids, int T) {
  pdl_entry();
  const unsigned long long epoch = ep_epoch(d);
  const int t = blockIdx.x, H = d.H, k = d.k, G = H / 64;
  if (t == 0 && threadIdx.x < d.world) ep_nrows(d, threadIdx.x)[d.rank] = T * k;
  if (t < T) {
    for (int j = 0; j < k; j++) {
      const int i = t * k + j;
      const int e = ids[i];
      const int own = min(max(e / d.E_loc, 0), d.world - 1);
      const size_t row = (size_t)d.rank * d.cap + i;
      uint8_t* dx = ep_rx(d, own) + row * H;
      const uint8_t* sx = xq + (size_t)t * xq_stride;
      for (int c = threadIdx.x; c < H / 16; c += blockDim.x)
        reinterpret_cast<uint4*>(dx)[c] = *reinterpret_cast<const uint4*>(sx + c * 16);
      uint8_t* ds = ep_rs(d, own) + row * G;
      const uint8_t* ss = xs + (size_t)t * xs_stride;
      for (int c = threadIdx.x; c < G / 4; c += blockDim.x)
        reinterpret_cast<uint32_t*>(ds)[c] = *reinterpret_cast<const uint32_t*>(ss + c * 4);
      if (threadIdx.x < d.world)
        ep_meta(d, threadIdx.x)[row] = (int)threadIdx.x == own ? e - own * d.E_loc : -1;
    }
  }
  ep_publish(d, epoch, 0);
}

}  // namespace moet

using namespace moet;

void ep_dispatch(torch::Tensor desc, torch::Tensor xq, torch::Tensor xs, torch::Tensor ids) {
  EpDesc d = ep_desc_from(desc);
  const int T = ids.size(0);
  TORCH_CHECK(ids.dim() == 2 && ids.size(1) == d.k && ids.is_contiguous() && ids.scalar_type() == at::kInt,
              "ep_dispatch: ids [T, k] int32");
  TORCH_CHECK((int64_t)T * d.k <= d.cap, "ep_dispatch: T * k exceeds the EP slab (", d.cap, " rows)");
  TORCH_CHECK(xq.size(1) == d.H && xq.stride(1) == 1 && (xq.stride(0) % 16) == 0 &&
              reinterpret_cast<uintptr_t>(xq.data_ptr()) % 16 == 0, "ep_dispatch: xq [T, H] 16-byte rows");
  TORCH_CHECK(xs.size(1) == d.H / 64 && xs.stride(1) == 1 && (xs.stride(0) % 4) == 0 &&
              reinterpret_cast<uintptr_t>(xs.data_ptr()) % 4 == 0, "ep_dispatch: xs [T, H/64]");
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(ep_dispatch_kernel, std::max(T, 1), 256, 0, stream, d, (const uint8_t*)xq.data_ptr(), xq.stride(0),
           (const uint8_t*)xs.data_ptr(), xs.stride(0), ids.data_ptr<int>(), T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Symmetric buffer size for (world, cap, H).
int64_t ep_buffer_bytes(int64_t world, int64_t cap, int64_t H) {
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  return 256 + al(world * cap * H) + al(world * cap * (H / 64)) + al(world * cap * 4) + cap * H * 4;
}
