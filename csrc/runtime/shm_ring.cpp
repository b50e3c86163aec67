// Host shared-memory broadcast ring: one producer, up to 16 consumers, variable-length records.
//
// The multi-GPU server's leader rank (rank 0: decoder and reaper) publishes every decoded task
// once; each tensor-parallel follower rank reads the same stream of records at its own pace. The
// ring lives in a POSIX shared-memory segment, so the transfer is one memcpy in and one memcpy out
// per consumer, with no pickling through a pipe per follower and no Python lock.
//
// Layout: a header (magic, capacity, consumer count, the producer's write position, one read
// position per consumer, a closed flag, one liveness word per consumer) followed by `capacity`
// data bytes (a power of two). Positions are monotonically increasing byte counters; a record is
// [u64 length][payload][pad to 8 bytes]; a record that would cross the end of the buffer is
// preceded by a wrap marker (length = ~0) and starts again at offset 0. The producer may reuse
// bytes only once every live consumer has read past them. Positions are 64-bit atomics in the
// shared segment (lock-free and address-free on the supported hosts), written with release and
// read with acquire ordering so a consumer that sees a new position also sees the bytes.
//
// Every wait is bounded by the caller's timeout; a consumer can be detached (declared dead), after
// which the producer no longer waits for it. The reference has no multi-process runtime; this is
// the host half of this build's multi-GPU serving.
#include <pybind11/pybind11.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace py = pybind11;

namespace {

constexpr uint64_t kMagic = 0x41505043524e4731ull;  // "APPCRNG1"
constexpr int kMaxConsumers = 16;
constexpr uint64_t kWrap = ~0ull;

struct alignas(64) Header {
  uint64_t magic;
  uint64_t capacity;
  uint32_t n_consumers;
  uint32_t pad0;
  alignas(64) std::atomic<uint64_t> head;
  alignas(64) std::atomic<uint64_t> tail[kMaxConsumers];
  alignas(64) std::atomic<uint32_t> closed;
  std::atomic<uint32_t> attached[kMaxConsumers];
};

static_assert(std::atomic<uint64_t>::is_always_lock_free, "64-bit atomics must be lock-free");

inline uint64_t pad8(uint64_t n) { return (n + 7) & ~7ull; }

class ShmRing {
 public:
  ShmRing(const std::string& name, uint64_t capacity, int n_consumers, bool create) : name_(name) {
    if (create) {
      if (capacity < 4096 || (capacity & (capacity - 1)) != 0)
        throw std::invalid_argument("shm ring: capacity must be a power of two >= 4096");
      if (n_consumers < 1 || n_consumers > kMaxConsumers)
        throw std::invalid_argument("shm ring: 1..16 consumers");
      fd_ = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
      if (fd_ < 0) throw std::runtime_error("shm ring: shm_open(create) failed for " + name);
      size_ = sizeof(Header) + capacity;
      if (ftruncate(fd_, static_cast<off_t>(size_)) != 0) {
        ::close(fd_);
        shm_unlink(name.c_str());
        throw std::runtime_error("shm ring: ftruncate failed");
      }
    } else {
      fd_ = shm_open(name.c_str(), O_RDWR, 0600);
      if (fd_ < 0) throw std::runtime_error("shm ring: shm_open(attach) failed for " + name);
      struct stat st;
      if (fstat(fd_, &st) != 0) throw std::runtime_error("shm ring: fstat failed");
      size_ = static_cast<uint64_t>(st.st_size);
    }
    void* p = mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd_, 0);
    if (p == MAP_FAILED) throw std::runtime_error("shm ring: mmap failed");
    hdr_ = static_cast<Header*>(p);
    data_ = static_cast<uint8_t*>(p) + sizeof(Header);
    if (create) {
      hdr_->capacity = capacity;
      hdr_->n_consumers = static_cast<uint32_t>(n_consumers);
      hdr_->head.store(0, std::memory_order_relaxed);
      for (int i = 0; i < kMaxConsumers; ++i) {
        hdr_->tail[i].store(0, std::memory_order_relaxed);
        hdr_->attached[i].store(i < n_consumers ? 1u : 0u, std::memory_order_relaxed);
      }
      hdr_->closed.store(0, std::memory_order_relaxed);
      std::atomic_thread_fence(std::memory_order_release);
      hdr_->magic = kMagic;
    } else {
      if (hdr_->magic != kMagic) throw std::runtime_error("shm ring: not an initialised ring: " + name);
    }
    cap_ = hdr_->capacity;
  }

  ~ShmRing() { release(); }

  void release() {
    if (hdr_ != nullptr) munmap(hdr_, size_);
    if (fd_ >= 0) ::close(fd_);
    hdr_ = nullptr;
    fd_ = -1;
  }

  void unlink() { shm_unlink(name_.c_str()); }

  int n_consumers() const { return static_cast<int>(hdr_->n_consumers); }
  uint64_t capacity() const { return cap_; }

  // Oldest position any attached consumer still needs.
  uint64_t min_tail() const {
    uint64_t m = hdr_->head.load(std::memory_order_acquire);
    for (uint32_t i = 0; i < hdr_->n_consumers; ++i)
      if (hdr_->attached[i].load(std::memory_order_acquire))
        m = std::min(m, hdr_->tail[i].load(std::memory_order_acquire));
    return m;
  }

  // Producer: append one record; false on timeout (no space) or when the ring is closed.
  bool push(const std::string& payload, double timeout_s) {
    const uint64_t need = 8 + pad8(payload.size());
    if (need + 8 > cap_) throw std::invalid_argument("shm ring: record larger than the ring");
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    uint64_t head = hdr_->head.load(std::memory_order_relaxed);
    const uint64_t off = head & (cap_ - 1);
    const uint64_t skip = (off + need > cap_) ? (cap_ - off) : 0;  // wrap: the rest of the buffer
    int spins = 0;
    while (head + skip + need - min_tail() > cap_) {
      if (hdr_->closed.load(std::memory_order_acquire)) return false;
      if (std::chrono::steady_clock::now() > deadline) return false;
      backoff(spins);
    }
    if (skip) {
      *reinterpret_cast<uint64_t*>(data_ + off) = kWrap;
      head += skip;
    }
    uint8_t* dst = data_ + (head & (cap_ - 1));
    const uint64_t n = payload.size();
    std::memcpy(dst, &n, 8);
    std::memcpy(dst + 8, payload.data(), n);
    hdr_->head.store(head + need, std::memory_order_release);
    return true;
  }

  // Consumer `c`: the next record, or None on timeout / after close with nothing left.
  py::object pop(int c, double timeout_s) {
    check_consumer(c);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    uint64_t tail = hdr_->tail[c].load(std::memory_order_relaxed);
    int spins = 0;
    while (true) {
      const uint64_t head = hdr_->head.load(std::memory_order_acquire);
      if (head != tail) break;
      if (hdr_->closed.load(std::memory_order_acquire)) return py::none();
      if (std::chrono::steady_clock::now() > deadline) return py::none();
      backoff(spins);
    }
    uint64_t off = tail & (cap_ - 1);
    uint64_t n;
    std::memcpy(&n, data_ + off, 8);
    if (n == kWrap) {
      tail += cap_ - off;
      off = 0;
      std::memcpy(&n, data_, 8);
    }
    std::string out(reinterpret_cast<const char*>(data_ + off + 8), n);
    hdr_->tail[c].store(tail + 8 + pad8(n), std::memory_order_release);
    return py::bytes(out);
  }

  // A consumer that died is no longer waited for (and one that rejoins resumes at the head).
  void detach(int c) {
    check_consumer(c);
    hdr_->attached[c].store(0, std::memory_order_release);
  }
  void attach(int c) {
    check_consumer(c);
    hdr_->tail[c].store(hdr_->head.load(std::memory_order_acquire), std::memory_order_release);
    hdr_->attached[c].store(1, std::memory_order_release);
  }
  bool attached(int c) const {
    check_consumer(c);
    return hdr_->attached[c].load(std::memory_order_acquire) != 0;
  }
  void close() { hdr_->closed.store(1, std::memory_order_release); }
  bool closed() const { return hdr_->closed.load(std::memory_order_acquire) != 0; }
  uint64_t head() const { return hdr_->head.load(std::memory_order_acquire); }
  uint64_t tail(int c) const {
    check_consumer(c);
    return hdr_->tail[c].load(std::memory_order_acquire);
  }

 private:
  void check_consumer(int c) const {
    if (c < 0 || c >= static_cast<int>(hdr_->n_consumers)) throw std::out_of_range("shm ring: bad consumer id");
  }
  static void backoff(int& spins) {
    if (++spins < 64) return;
    if (spins < 256) {
      std::this_thread::yield();
      return;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }

  std::string name_;
  int fd_ = -1;
  uint64_t size_ = 0;
  uint64_t cap_ = 0;
  Header* hdr_ = nullptr;
  uint8_t* data_ = nullptr;
};

}  // namespace

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "appcorr_b200 host runtime: shared-memory broadcast ring for multi-rank serving";
  py::class_<ShmRing>(m, "ShmRing")
      .def(py::init<const std::string&, uint64_t, int, bool>(), py::arg("name"), py::arg("capacity") = 1 << 26,
           py::arg("n_consumers") = 1, py::arg("create") = false)
      .def("push",
           [](ShmRing& r, py::bytes b, double timeout_s) {
             std::string s = b;
             py::gil_scoped_release nogil;
             return r.push(s, timeout_s);
           },
           py::arg("payload"), py::arg("timeout_s") = 10.0)
      .def("pop",
           [](ShmRing& r, int c, double timeout_s) -> py::object {
             // wait without the GIL, then build the bytes object with it
             {
               py::gil_scoped_release nogil;
               const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
               while (r.head() == r.tail(c) && !r.closed() && std::chrono::steady_clock::now() < deadline)
                 std::this_thread::sleep_for(std::chrono::microseconds(20));
             }
             return r.pop(c, 0.0);
           },
           py::arg("consumer"), py::arg("timeout_s") = 10.0)
      .def("detach", &ShmRing::detach)
      .def("attach", &ShmRing::attach)
      .def("attached", &ShmRing::attached)
      .def("close", &ShmRing::close)
      .def("closed", &ShmRing::closed)
      .def("release", &ShmRing::release)
      .def("unlink", &ShmRing::unlink)
      .def_property_readonly("n_consumers", &ShmRing::n_consumers)
      .def_property_readonly("capacity", &ShmRing::capacity)
      .def_property_readonly("head", &ShmRing::head)
      .def("tail", &ShmRing::tail);
}
