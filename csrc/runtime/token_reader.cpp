// Native token-window reader for the pretraining data path
// (module nano_qwen_b200._runtime).
//
// Memory-maps every token shard once (read-only, MADV_RANDOM) and serves
// windows [start, start+n) of the virtual concatenation as int64 arrays.  The
// copy/widening runs without the GIL, so DataLoader worker threads overlap, and
// a window that spans shard boundaries is gathered without Python-level
// slicing.  Tokens past the end are filled with `pad`.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace {

struct Shard {
  const uint8_t* base = nullptr;
  size_t bytes = 0;
  int64_t tokens = 0;
};

class TokenWindowReader {
 public:
  TokenWindowReader(const std::vector<std::string>& files, int itemsize, int64_t pad)
      : itemsize_(itemsize), pad_(pad) {
    if (itemsize != 2 && itemsize != 4 && itemsize != 8)
      throw std::invalid_argument("TokenWindowReader: itemsize must be 2, 4 or 8");
    starts_.push_back(0);
    for (const auto& f : files) {
      const int fd = ::open(f.c_str(), O_RDONLY);
      if (fd < 0) throw std::runtime_error("TokenWindowReader: cannot open " + f);
      struct stat st {};
      if (::fstat(fd, &st) != 0) {
        ::close(fd);
        throw std::runtime_error("TokenWindowReader: cannot stat " + f);
      }
      Shard s;
      s.bytes = static_cast<size_t>(st.st_size);
      s.tokens = static_cast<int64_t>(s.bytes / itemsize);
      if (s.bytes > 0) {
        void* p = ::mmap(nullptr, s.bytes, PROT_READ, MAP_SHARED, fd, 0);
        if (p == MAP_FAILED) {
          ::close(fd);
          throw std::runtime_error("TokenWindowReader: mmap failed for " + f);
        }
        ::madvise(p, s.bytes, MADV_RANDOM);
        s.base = static_cast<const uint8_t*>(p);
      }
      ::close(fd);
      shards_.push_back(s);
      starts_.push_back(starts_.back() + s.tokens);
    }
  }

  ~TokenWindowReader() {
    for (auto& s : shards_)
      if (s.base != nullptr) ::munmap(const_cast<uint8_t*>(s.base), s.bytes);
  }

  int64_t total_tokens() const { return starts_.back(); }

  py::array_t<int64_t> read(int64_t start, int64_t n) const {
    if (start < 0 || n < 0) throw std::invalid_argument("TokenWindowReader.read: negative range");
    py::array_t<int64_t> out(n);
    int64_t* dst = out.mutable_data();
    {
      py::gil_scoped_release nogil;
      fill(start, n, dst);
    }
    return out;
  }

 private:
  void fill(int64_t start, int64_t n, int64_t* dst) const {
    int64_t filled = 0;
    auto it = std::upper_bound(starts_.begin(), starts_.end(), start);
    size_t f = static_cast<size_t>(std::max<std::ptrdiff_t>(0, (it - starts_.begin()) - 1));
    int64_t pos = start;
    while (filled < n && f < shards_.size()) {
      const Shard& s = shards_[f];
      const int64_t local = pos - starts_[f];
      if (local >= s.tokens) { ++f; continue; }
      const int64_t take = std::min(n - filled, s.tokens - local);
      const uint8_t* src = s.base + static_cast<size_t>(local) * itemsize_;
      switch (itemsize_) {
        case 2: widen(reinterpret_cast<const uint16_t*>(src), take, dst + filled); break;
        case 4: widen(reinterpret_cast<const uint32_t*>(src), take, dst + filled); break;
        default: std::memcpy(dst + filled, src, static_cast<size_t>(take) * 8); break;
      }
      filled += take;
      pos += take;
      ++f;
    }
    for (; filled < n; ++filled) dst[filled] = pad_;
  }

  template <typename T>
  static void widen(const T* src, int64_t n, int64_t* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = static_cast<int64_t>(src[i]);
  }

  int itemsize_;
  int64_t pad_;
  std::vector<Shard> shards_;
  std::vector<int64_t> starts_;
};

}  // namespace

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "nano_qwen_b200 native host runtime (token-window reader)";
  py::class_<TokenWindowReader>(m, "TokenWindowReader")
      .def(py::init<const std::vector<std::string>&, int, int64_t>(), py::arg("files"),
           py::arg("itemsize"), py::arg("pad") = 0)
      .def("read", &TokenWindowReader::read, py::arg("start"), py::arg("n"))
      .def_property_readonly("total_tokens", &TokenWindowReader::total_tokens);
}
