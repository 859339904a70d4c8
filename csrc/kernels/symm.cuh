// Tensor-parallel all-reduce fused into the producing and consuming kernels,
// over peer (NVLink / NVSwitch) memory.
//
// Every rank owns one symmetric buffer (cudaMalloc'd, exported by CUDA IPC and
// mapped into every peer):
//     [flags: u64 x kMaxTP][pad to 256 B][recv: 2 parities x W sources x cap f32]
// Producer side (the epilogue of a row-parallel GEMV, or of the expert combine):
// each CTA stores its fp32 partial tile straight into slot [parity][rank] of
// EVERY rank's recv area (peer stores), then arrives on a local counter; the
// last CTA of the grid publishes epoch = ncall + 1 into flag[rank] of every
// peer with a system-scope release.
// Consumer side (the prologue of the next RMSNorm): one thread per CTA waits
// (bounded) until flag[r] >= epoch for all r, then every thread sums the W
// partials in rank order 0..W-1 (so all ranks produce bit-identical sums) plus
// the residual.  The consumer's last CTA advances ncall.
// Parities alternate per call: a peer can run at most one reduction ahead of
// this rank (its next consumer waits on this rank's next producer), so the
// parity it writes next is never the one being read here.
#pragma once
#include "common.cuh"

namespace moet {

constexpr int kMaxTP = 8;
constexpr int kSymmFlagBytes = 256;

struct ArDesc {
  float* recv[kMaxTP];               // rank p's recv area (parity 0, source 0)
  unsigned long long* flag[kMaxTP];  // rank p's flag array [kMaxTP]
  unsigned long long* ncall;         // local: number of completed reductions
  unsigned int* arrive;              // local: producer CTA arrivals (self-resetting)
  unsigned int* done;                // local: consumer CTA completions (self-resetting)
  int* status;
  long long cap;                     // floats per (parity, source) slot
  int rank, world;
  long long spin_limit;              // bounded wait: polls before giving up
};

MOET_DEVICE unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

MOET_DEVICE void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

MOET_DEVICE unsigned long long ar_epoch(const ArDesc& d) {
  return *reinterpret_cast<volatile unsigned long long*>(d.ncall) + 1ull;
}

// Slot base of source `src` at parity of `epoch` in rank p's recv area.
MOET_DEVICE float* ar_slot(const ArDesc& d, int p, unsigned long long epoch, int src) {
  return d.recv[p] + ((long long)((epoch - 1ull) & 1ull) * d.world + src) * d.cap;
}

// Producer: called by every thread of the CTA after its peer stores (or by
// the only storing warp when `warp_only`).  The last CTA of the grid publishes.
MOET_DEVICE void ar_producer_arrive(const ArDesc& d, unsigned long long epoch, bool warp_only = false) {
  if (warp_only) __syncwarp(); else __syncthreads();
  if ((warp_only ? (threadIdx.x & 31) : threadIdx.x) != 0) return;
  const unsigned total = gridDim.x * gridDim.y * gridDim.z;
  __threadfence_system();
  const unsigned prev = atomicAdd(d.arrive, 1u);
  if (prev != total - 1) return;
  *d.arrive = 0u;                      // every CTA has arrived: reset for the next call
  __threadfence_system();
  for (int p = 0; p < d.world; p++) st_release_sys_u64(d.flag[p] + d.rank, epoch);
}

// Consumer: wait for all W producers of `epoch`.  Returns false (and records
// kTimeout) if the bounded wait ran out or an earlier wait already failed.
MOET_DEVICE bool ar_consumer_wait(const ArDesc& d, unsigned long long epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = (d.status == nullptr || *reinterpret_cast<volatile int*>(d.status) == 0);
    const unsigned long long* f = d.flag[d.rank];
    for (int r = 0; r < d.world && good; r++) {
      long long n = 0;
      while (ld_acquire_sys_u64(f + r) < epoch) {
        if (++n > d.spin_limit) { good = 0; set_status(d.status, kTimeout); break; }
        __nanosleep(64);
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

// Consumer: called by every thread after its last read of the recv slots.
MOET_DEVICE void ar_consumer_done(const ArDesc& d) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  const unsigned total = gridDim.x * gridDim.y * gridDim.z;
  __threadfence();
  if (atomicAdd(d.done, 1u) == total - 1) {
    *d.done = 0u;
    *d.ncall = *d.ncall + 1ull;
    __threadfence();
  }
}

}  // namespace moet

// Host side: the descriptor travels from Python as a CPU int64 tensor
//   [world, rank, cap, spin_limit, ncall, arrive, done, status, recv x 8, flag x 8].
#include <ATen/core/Tensor.h>
#include <c10/util/Exception.h>
namespace moet {
constexpr int kArDescLen = 8 + 2 * kMaxTP;
inline ArDesc ar_desc_from(const at::Tensor& t) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.numel() == kArDescLen,
              "all-reduce descriptor: CPU int64 tensor of ", kArDescLen);
  const int64_t* v = t.data_ptr<int64_t>();
  ArDesc d{};
  d.world = (int)v[0]; d.rank = (int)v[1]; d.cap = v[2]; d.spin_limit = v[3];
  TORCH_CHECK(d.world >= 1 && d.world <= kMaxTP && d.rank >= 0 && d.rank < d.world, "all-reduce descriptor: rank/world");
  d.ncall = reinterpret_cast<unsigned long long*>(v[4]);
  d.arrive = reinterpret_cast<unsigned int*>(v[5]);
  d.done = reinterpret_cast<unsigned int*>(v[6]);
  d.status = reinterpret_cast<int*>(v[7]);
  for (int p = 0; p < kMaxTP; p++) {
    d.recv[p] = reinterpret_cast<float*>(v[8 + p]);
    d.flag[p] = reinterpret_cast<unsigned long long*>(v[8 + kMaxTP + p]);
  }
  for (int p = 0; p < d.world; p++) TORCH_CHECK(d.recv[p] && d.flag[p], "all-reduce descriptor: null peer pointer");
  return d;
}
}  // namespace moet
