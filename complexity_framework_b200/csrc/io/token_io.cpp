// Native token-shard reader: memory-maps a flat token file (uint16 or uint32
// ids) and gathers fixed-length windows into (pinned) host tensors with
// several threads and without holding the Python interpreter lock, so batch
// assembly overlaps the GPU step.  Also computes token-frequency histograms
// over a range of the shard.
//
// Counterpart of the numpy memmap slicing in
// complexity/data/token_shards.py:196-215 (load) and :333-370 (per-sample
// window reads inside TokenShardDataset.__iter__), and of the frequency
// pass :216-262.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <torch/extension.h>

namespace {

class ShardReader {
 public:
  ShardReader(const std::string& path, int64_t elem_bytes, int64_t num_tokens)
      : path_(path), elem_(elem_bytes), n_(num_tokens) {
    if (elem_ != 2 && elem_ != 4) throw std::invalid_argument("token width must be 2 or 4 bytes");
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (::fstat(fd_, &st) != 0) {
      ::close(fd_);
      throw std::runtime_error("cannot stat " + path);
    }
    bytes_ = static_cast<size_t>(st.st_size);
    if (static_cast<size_t>(n_) * elem_ > bytes_) {
      ::close(fd_);
      throw std::runtime_error("token file shorter than its index says");
    }
    if (bytes_ > 0) {
      base_ = ::mmap(nullptr, bytes_, PROT_READ, MAP_SHARED, fd_, 0);
      if (base_ == MAP_FAILED) {
        ::close(fd_);
        throw std::runtime_error("mmap failed for " + path);
      }
      ::madvise(base_, bytes_, MADV_RANDOM);
    }
  }
  ~ShardReader() {
    if (base_ && base_ != MAP_FAILED) ::munmap(base_, bytes_);
    if (fd_ >= 0) ::close(fd_);
  }

  int64_t size() const { return n_; }
  int64_t elem_bytes() const { return elem_; }

  // out[b, :] = tokens[pos[b] : pos[b] + out.size(1)]
  void gather(const torch::Tensor& pos, torch::Tensor out, int64_t threads) const {
    TORCH_CHECK(pos.dim() == 1 && pos.scalar_type() == torch::kLong && pos.device().is_cpu(),
                "positions must be a 1-D CPU int64 tensor");
    TORCH_CHECK(out.dim() == 2 && out.is_contiguous() && out.device().is_cpu() &&
                    (out.scalar_type() == torch::kLong || out.scalar_type() == torch::kInt),
                "out must be a contiguous CPU [B, L] int64/int32 tensor");
    TORCH_CHECK(out.size(0) == pos.size(0), "one position per row");
    const int64_t B = out.size(0), L = out.size(1);
    const int64_t* p = pos.data_ptr<int64_t>();
    for (int64_t b = 0; b < B; ++b)
      TORCH_CHECK(p[b] >= 0 && p[b] + L <= n_, "window [", p[b], ", ", p[b] + L,
                  ") outside the shard of ", n_, " tokens");
    const bool o64 = out.scalar_type() == torch::kLong;
    void* o = out.data_ptr();
    auto work = [&](int64_t b0, int64_t b1) {
      for (int64_t b = b0; b < b1; ++b) {
        const int64_t s = p[b];
        if (elem_ == 2) {
          const uint16_t* src = static_cast<const uint16_t*>(base_) + s;
          if (o64) {
            int64_t* d = static_cast<int64_t*>(o) + b * L;
            for (int64_t i = 0; i < L; ++i) d[i] = src[i];
          } else {
            int32_t* d = static_cast<int32_t*>(o) + b * L;
            for (int64_t i = 0; i < L; ++i) d[i] = src[i];
          }
        } else {
          const uint32_t* src = static_cast<const uint32_t*>(base_) + s;
          if (o64) {
            int64_t* d = static_cast<int64_t*>(o) + b * L;
            for (int64_t i = 0; i < L; ++i) d[i] = src[i];
          } else {
            int32_t* d = static_cast<int32_t*>(o) + b * L;
            for (int64_t i = 0; i < L; ++i) d[i] = static_cast<int32_t>(src[i]);
          }
        }
      }
    };
    run_parallel(B, threads, work);
  }

  // counts[v] = occurrences of token v in [start, end); ids >= vocab are
  // counted in counts[vocab] (one overflow bin).
  torch::Tensor frequencies(int64_t vocab, int64_t start, int64_t end, int64_t threads) const {
    TORCH_CHECK(vocab > 0 && start >= 0 && end <= n_ && start <= end, "bad frequency range");
    const int64_t T = std::max<int64_t>(1, std::min<int64_t>(threads, 64));
    std::vector<std::vector<int64_t>> part(T, std::vector<int64_t>(vocab + 1, 0));
    const int64_t n = end - start;
    auto work = [&](int64_t t) {
      const int64_t a = start + n * t / T, b = start + n * (t + 1) / T;
      auto& c = part[t];
      if (elem_ == 2) {
        const uint16_t* src = static_cast<const uint16_t*>(base_);
        for (int64_t i = a; i < b; ++i) c[std::min<int64_t>(src[i], vocab)]++;
      } else {
        const uint32_t* src = static_cast<const uint32_t*>(base_);
        for (int64_t i = a; i < b; ++i) c[std::min<int64_t>(src[i], vocab)]++;
      }
    };
    std::vector<std::thread> ts;
    for (int64_t t = 1; t < T; ++t) ts.emplace_back(work, t);
    work(0);
    for (auto& th : ts) th.join();
    auto out = torch::zeros({vocab + 1}, torch::kLong);
    int64_t* o = out.data_ptr<int64_t>();
    for (auto& c : part)
      for (int64_t v = 0; v <= vocab; ++v) o[v] += c[v];
    return out;
  }

 private:
  template <typename F>
  static void run_parallel(int64_t rows, int64_t threads, F&& fn) {
    const int64_t T = std::max<int64_t>(1, std::min<int64_t>(threads, rows));
    if (T == 1) {
      fn(0, rows);
      return;
    }
    std::vector<std::thread> ts;
    for (int64_t t = 1; t < T; ++t) ts.emplace_back(fn, rows * t / T, rows * (t + 1) / T);
    fn(0, rows / T);
    for (auto& th : ts) th.join();
  }

  std::string path_;
  int64_t elem_;
  int64_t n_;
  int fd_ = -1;
  size_t bytes_ = 0;
  void* base_ = nullptr;
};

// Pack variable-length documents (concatenated ids + offsets) into rows of
// `seq_len` tokens, greedy first-fit in input order, documents longer than a
// row are split.  Returns (tokens [R, seq_len], doc_ids [R, seq_len]) with
// `pad_id` / -1 in the unused tail.
std::vector<torch::Tensor> pack_documents(const torch::Tensor& ids, const torch::Tensor& offsets,
                                          int64_t seq_len, int64_t pad_id) {
  TORCH_CHECK(ids.dim() == 1 && ids.scalar_type() == torch::kLong, "ids: 1-D int64");
  TORCH_CHECK(offsets.dim() == 1 && offsets.scalar_type() == torch::kLong, "offsets: 1-D int64");
  TORCH_CHECK(seq_len > 0, "seq_len must be positive");
  const int64_t* x = ids.data_ptr<int64_t>();
  const int64_t* off = offsets.data_ptr<int64_t>();
  const int64_t D = offsets.size(0) - 1;
  std::vector<std::vector<int64_t>> rows_t, rows_d;
  std::vector<int64_t> fill;
  for (int64_t d = 0; d < D; ++d) {
    int64_t a = off[d];
    const int64_t e = off[d + 1];
    while (a < e) {
      const int64_t len = std::min<int64_t>(e - a, seq_len);
      int64_t r = -1;
      for (size_t i = 0; i < fill.size(); ++i)
        if (seq_len - fill[i] >= len) {
          r = static_cast<int64_t>(i);
          break;
        }
      if (r < 0) {
        rows_t.emplace_back(seq_len, pad_id);
        rows_d.emplace_back(seq_len, -1);
        fill.push_back(0);
        r = static_cast<int64_t>(fill.size()) - 1;
      }
      for (int64_t i = 0; i < len; ++i) {
        rows_t[r][fill[r] + i] = x[a + i];
        rows_d[r][fill[r] + i] = d;
      }
      fill[r] += len;
      a += len;
    }
  }
  const int64_t R = static_cast<int64_t>(rows_t.size());
  auto T = torch::empty({R, seq_len}, torch::kLong);
  auto Dd = torch::empty({R, seq_len}, torch::kLong);
  for (int64_t r = 0; r < R; ++r) {
    std::memcpy(T.data_ptr<int64_t>() + r * seq_len, rows_t[r].data(), seq_len * 8);
    std::memcpy(Dd.data_ptr<int64_t>() + r * seq_len, rows_d[r].data(), seq_len * 8);
  }
  return {T, Dd};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "complexity_framework_b200 native data IO";
  py::class_<ShardReader>(m, "ShardReader")
      .def(py::init<const std::string&, int64_t, int64_t>(), py::arg("path"),
           py::arg("elem_bytes"), py::arg("num_tokens"))
      .def("size", &ShardReader::size)
      .def("elem_bytes", &ShardReader::elem_bytes)
      .def("gather", &ShardReader::gather, py::arg("positions"), py::arg("out"),
           py::arg("threads") = 4, py::call_guard<py::gil_scoped_release>())
      .def("frequencies", &ShardReader::frequencies, py::arg("vocab"), py::arg("start"),
           py::arg("end"), py::arg("threads") = 8, py::call_guard<py::gil_scoped_release>());
  m.def("pack_documents", &pack_documents, py::arg("ids"), py::arg("offsets"),
        py::arg("seq_len"), py::arg("pad_id") = 0);
}
