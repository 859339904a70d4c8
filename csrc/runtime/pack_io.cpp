// Native I/O for expert pack files: rows of `slot_bytes` at offset row * stride
// (stride a multiple of 4 KiB, so the same file serves buffered and O_DIRECT
// readers).  Reads run on a small thread pool with pread into caller-provided
// (pinned) host memory; every row reports its own status, so a failed read is
// never published by the caller.  Writes are pwrite + fdatasync.
//
// The read path of the reference's MmapPackStore / TieredPackStore
// (moe_w2_store.py, patch P:13086-13680) is Python preadv on a thread pool;
// here it is C++ so that a miss burst of hundreds of rows is one call.
#include <torch/extension.h>

#include <atomic>
#include <cerrno>
#include <cstring>
#include <fcntl.h>
#include <mutex>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

constexpr int64_t kAlign = 4096;

class PackFile {
 public:
  PackFile(const std::string& path, bool writable, bool direct, int64_t stride, int64_t threads)
      : path_(path), stride_(stride), threads_(std::max<int64_t>(1, threads)), direct_(direct) {
    TORCH_CHECK(stride > 0 && stride % kAlign == 0, "PackFile: stride must be a positive multiple of 4096");
    int flags = writable ? (O_RDWR | O_CREAT) : O_RDONLY;
    fd_ = ::open(path.c_str(), flags | O_CLOEXEC, 0644);
    TORCH_CHECK(fd_ >= 0, "PackFile: cannot open ", path, ": ", std::strerror(errno));
    if (direct) {
      dfd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);
      if (dfd_ < 0) direct_ = false;   // filesystem without O_DIRECT (tmpfs): buffered reads
    }
  }
  ~PackFile() { close(); }

  void close() {
    if (dfd_ >= 0) { ::close(dfd_); dfd_ = -1; }
    if (fd_ >= 0) { ::close(fd_); fd_ = -1; }
  }

  bool direct() const { return direct_; }
  int64_t stride() const { return stride_; }

  // rows: uint8 CPU [n, nbytes] written at row indices first_row + i.
  void write_rows(int64_t first_row, at::Tensor rows) {
    TORCH_CHECK(fd_ >= 0, "PackFile closed");
    TORCH_CHECK(rows.device().is_cpu() && rows.scalar_type() == at::kByte && rows.dim() == 2 && rows.is_contiguous(),
                "write_rows: contiguous uint8 CPU [n, bytes]");
    const int64_t n = rows.size(0), nb = rows.size(1);
    TORCH_CHECK(nb <= stride_, "write_rows: row larger than the stride");
    const uint8_t* p = rows.data_ptr<uint8_t>();
    for (int64_t i = 0; i < n; i++) {
      int64_t off = (first_row + i) * stride_, done = 0;
      while (done < nb) {
        ssize_t w = ::pwrite(fd_, p + i * nb + done, nb - done, off + done);
        TORCH_CHECK(w > 0 || errno == EINTR, "pwrite failed: ", std::strerror(errno));
        if (w > 0) done += w;
      }
    }
  }

  void sync() {
    TORCH_CHECK(fd_ >= 0, "PackFile closed");
    TORCH_CHECK(::fdatasync(fd_) == 0, "fdatasync failed: ", std::strerror(errno));
  }

  // Reads rows[i] into dst + i * dst_stride (nbytes each).  Returns per-row
  // status: 0 ok, else an errno value.  With O_DIRECT the destination rows and
  // the length must be 4 KiB aligned (the stride is); otherwise buffered reads.
  std::vector<int64_t> read_rows(std::vector<int64_t> rows, int64_t dst_ptr, int64_t dst_stride, int64_t nbytes) {
    TORCH_CHECK(fd_ >= 0, "PackFile closed");
    TORCH_CHECK(nbytes > 0 && nbytes <= stride_, "read_rows: nbytes");
    const int64_t n = rows.size();
    std::vector<int64_t> status(n, 0);
    if (n == 0) return status;
    uint8_t* dst = reinterpret_cast<uint8_t*>(dst_ptr);
    const bool use_direct = direct_ && dst_ptr % kAlign == 0 && dst_stride % kAlign == 0;
    std::atomic<int64_t> next{0};
    auto worker = [&]() {
      for (;;) {
        const int64_t i = next.fetch_add(1);
        if (i >= n) return;
        status[i] = read_one(rows[i], dst + i * dst_stride, nbytes, use_direct);
      }
    };
    const int64_t nt = std::min<int64_t>(threads_, n);
    std::vector<std::thread> pool;
    for (int64_t t = 1; t < nt; t++) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    return status;
  }

  // Host-side fault injection for tests: every `every`-th read (counted across
  // calls) fails with EIO.  0 disables.
  void inject_read_faults(int64_t every) { fault_every_ = every; reads_ = 0; }

  int64_t size_bytes() const {
    struct stat st;
    return ::fstat(fd_, &st) == 0 ? (int64_t)st.st_size : -1;
  }

 private:
  int64_t read_one(int64_t row, uint8_t* dst, int64_t nbytes, bool use_direct) {
    if (fault_every_ > 0 && (reads_.fetch_add(1) + 1) % fault_every_ == 0) return EIO;
    const int fd = use_direct ? dfd_ : fd_;
    const int64_t len = use_direct ? stride_ : nbytes;   // O_DIRECT reads whole aligned rows
    const int64_t off = row * stride_;
    int64_t done = 0;
    while (done < len) {
      ssize_t r = ::pread(fd, dst + done, len - done, off + done);
      if (r < 0) {
        if (errno == EINTR) continue;
        return errno;
      }
      if (r == 0) break;   // past EOF (a hole at the end): the rest reads as zeros
      done += r;
    }
    if (done < nbytes) std::memset(dst + done, 0, nbytes - done);
    return 0;
  }

  std::string path_;
  int64_t stride_;
  int64_t threads_;
  bool direct_;
  int fd_ = -1, dfd_ = -1;
  int64_t fault_every_ = 0;
  std::atomic<int64_t> reads_{0};
};

// Pinned (page-locked) host buffer of `bytes`, page aligned, as a uint8 tensor.
at::Tensor alloc_pinned_aligned(int64_t bytes) {
  return at::empty({bytes}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
}

}  // namespace

void register_pack_io(pybind11::module& m) {
  pybind11::class_<PackFile>(m, "PackFile")
      .def(pybind11::init<const std::string&, bool, bool, int64_t, int64_t>(), pybind11::arg("path"),
           pybind11::arg("writable"), pybind11::arg("direct"), pybind11::arg("stride"), pybind11::arg("threads") = 8)
      .def("write_rows", &PackFile::write_rows)
      .def("sync", &PackFile::sync)
      .def("read_rows", &PackFile::read_rows, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("inject_read_faults", &PackFile::inject_read_faults)
      .def("size_bytes", &PackFile::size_bytes)
      .def("close", &PackFile::close)
      .def_property_readonly("direct", &PackFile::direct)
      .def_property_readonly("stride", &PackFile::stride);
  m.def("alloc_pinned_aligned", &alloc_pinned_aligned);
}
