// Expert-parallel all-to-all over peer (NVLink / NVSwitch) memory for decode-sized
// MoE layers: data-parallel attention, routed experts partitioned over the ranks.
//
// Every rank owns one symmetric buffer (cudaMalloc'd, exported by CUDA IPC, mapped
// into every peer).  Layout, W ranks, cap routed rows per source, hidden H:
//   [flags u64: dispatch-from-src x 8 | return-from-owner x 8][n_rows int x 8] (256 B)
//   rx   [W][cap][H]      u8  e4m3 activation rows received from each source
//   rs   [W][cap][H/64]   u8  their UE8M0 per-64 scales
//   meta [W][cap]         i32 local expert id of the row, -1 if not routed here
//   ret  [cap][H]         f32 expert outputs of this rank's own routings, row t*k + j
// One MoE layer:
//   dispatch   (source)  row (t, j) -> owner's rx/rs/meta[src][t*k + j]; n_rows; epoch flag
//   recv_pairs (owner)   bounded wait for every source's flag, expert pair list of the rows
//   w13 GEMV -> SwiGLU -> w2 GEMV whose epilogue stores each output row straight into the
//              source's ret[t*k + j] and publishes a return flag to every source
//   combine    (source)  bounded wait for every owner, weighted sum in slot order 0..k-1
// The epoch of a layer is ncall + 1; the combine's last CTA advances ncall.  A slab is
// rewritten by the next layer's dispatch only after this rank's combine consumed the
// returns -- which every owner sends after reading the slab -- so one buffer suffices.
#pragma once
#include "common.cuh"

namespace moet {

constexpr int kEpMax = 8;

struct EpDesc {
  uint8_t* base[kEpMax];             // rank p's symmetric buffer
  unsigned long long* ncall;         // local: completed EP layers
  unsigned int* arrive;              // local: producer CTA arrivals (self-resetting)
  unsigned int* done;                // local: combine CTA completions (self-resetting)
  int* status;
  int rank, world, cap, H, E_loc, k;
  long long spin_limit;
};

MOET_DEVICE size_t ep_align(size_t x) { return (x + 255) & ~size_t(255); }
MOET_DEVICE unsigned long long* ep_flags(const EpDesc& d, int p) { return reinterpret_cast<unsigned long long*>(d.base[p]); }
MOET_DEVICE int* ep_nrows(const EpDesc& d, int p) { return reinterpret_cast<int*>(d.base[p] + 128); }
MOET_DEVICE uint8_t* ep_rx(const EpDesc& d, int p) { return d.base[p] + 256; }
MOET_DEVICE uint8_t* ep_rs(const EpDesc& d, int p) {
  return d.base[p] + 256 + ep_align((size_t)d.world * d.cap * d.H);
}
MOET_DEVICE int* ep_meta(const EpDesc& d, int p) {
  return reinterpret_cast<int*>(ep_rs(d, p) + ep_align((size_t)d.world * d.cap * (d.H / 64)));
}
MOET_DEVICE float* ep_ret(const EpDesc& d, int p) {
  return reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ep_meta(d, p)) + ep_align((size_t)d.world * d.cap * 4));
}
MOET_DEVICE unsigned long long ep_epoch(const EpDesc& d) {
  return *reinterpret_cast<volatile unsigned long long*>(d.ncall) + 1ull;
}

MOET_DEVICE unsigned long long ep_ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
MOET_DEVICE void ep_st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Producer side: every thread of every CTA calls it after its peer stores; the last CTA
// of the grid publishes `epoch` into flag slot [which * kEpMax + rank] of every rank.
MOET_DEVICE void ep_publish(const EpDesc& d, unsigned long long epoch, int which) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  const unsigned total = gridDim.x * gridDim.y * gridDim.z;
  __threadfence_system();
  if (atomicAdd(d.arrive, 1u) != total - 1) return;
  *d.arrive = 0u;
  __threadfence_system();
  for (int p = 0; p < d.world; p++) ep_st_release(ep_flags(d, p) + which * kEpMax + d.rank, epoch);
}

// Consumer side: bounded wait until flag [which * kEpMax + src] >= epoch for every src.
// False (and kTimeout recorded) if the wait ran out or an earlier wait already failed.
MOET_DEVICE bool ep_wait(const EpDesc& d, unsigned long long epoch, int which) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = d.status == nullptr || *reinterpret_cast<volatile int*>(d.status) == 0;
    const unsigned long long* f = ep_flags(d, d.rank) + which * kEpMax;
    for (int r = 0; r < d.world && good; r++) {
      long long n = 0;
      while (ep_ld_acquire(f + r) < epoch) {
        if (++n > d.spin_limit) { good = 0; set_status(d.status, kTimeout); break; }
        __nanosleep(64);
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

}  // namespace moet

// Host side: the descriptor travels from Python as a CPU int64 tensor
//   [world, rank, cap, H, E_loc, k, spin_limit, ncall, arrive, done, status, base x 8].
#include <ATen/core/Tensor.h>
#include <c10/util/Exception.h>
namespace moet {
constexpr int kEpDescLen = 11 + kEpMax;
inline EpDesc ep_desc_from(const at::Tensor& t) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.numel() == kEpDescLen,
              "EP descriptor: CPU int64 tensor of ", kEpDescLen);
  const int64_t* v = t.data_ptr<int64_t>();
  EpDesc d{};
  d.world = (int)v[0]; d.rank = (int)v[1]; d.cap = (int)v[2]; d.H = (int)v[3]; d.E_loc = (int)v[4]; d.k = (int)v[5];
  d.spin_limit = v[6];
  d.ncall = reinterpret_cast<unsigned long long*>(v[7]);
  d.arrive = reinterpret_cast<unsigned int*>(v[8]);
  d.done = reinterpret_cast<unsigned int*>(v[9]);
  d.status = reinterpret_cast<int*>(v[10]);
  TORCH_CHECK(d.world >= 1 && d.world <= kEpMax && d.rank >= 0 && d.rank < d.world && d.H % 64 == 0 && d.cap > 0,
              "EP descriptor: rank / world / H / cap");
  for (int p = 0; p < kEpMax; p++) d.base[p] = reinterpret_cast<uint8_t*>(v[11 + p]);
  for (int p = 0; p < d.world; p++) TORCH_CHECK(d.base[p] != nullptr, "EP descriptor: null peer buffer");
  return d;
}
}  // namespace moet
