// Host-side native runtime pieces (module `_host`, plain C++17, no CUDA):
//
//   BlockAllocator : paged-KV block bookkeeping (free list + per-slot block lists), the engine's allocator.
//   quantize_groups / dequantize_groups : per-128-element absmax quantization to 8, 6 or 5-bit signed codes
//                    (6/5-bit codes bit-packed), the payload format of the reference's quantized all-reduce
//                    (dotsnote/engine/arcstats_pkg/arcstats/host_ar.py:47-54, csrc/host_arc.c:169 group512).
//   HostReducer    : multi-threaded CPU reduction of W ranks' quantized contributions: dequantize, sum in rank
//                    order with fp32 (no FMA contraction, so the result is independent of vector width and
//                    thread count), requantize to the result bit width. The reference runs this as its
//                    CPU-reduced all-reduce (csrc/host_arc.c:1-21, worker :299, arc_reduce_all :381); here it
//                    is the exactness oracle for quantized reductions and the host path for GPUs without
//                    peer access.
//   StepLog        : buffered binary log of fixed-width int64 records (the reference's steplog.py format:
//                    a header with the field count, then records), flushed on close.
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace py = pybind11;

// ------------------------------------------------------------------------------------------ allocator
class BlockAllocator {
 public:
  BlockAllocator(int64_t n_blocks, int64_t n_slots) : n_blocks_(n_blocks), owned_(n_slots) {
    if (n_blocks < 0 || n_slots < 0) throw std::invalid_argument("negative size");
    free_.reserve(n_blocks);
    for (int64_t b = n_blocks - 1; b >= 0; --b) free_.push_back((int32_t)b);
  }
  int64_t n_free() const { return (int64_t)free_.size(); }
  int64_t n_blocks_of(int64_t slot) const { return (int64_t)at(slot).size(); }
  std::vector<int32_t> blocks_of(int64_t slot) const { return at(slot); }
  std::vector<int32_t> allocate(int64_t slot, int64_t n) {
    auto& o = at(slot);
    if (n < 0) throw std::invalid_argument("negative block count");
    if ((int64_t)free_.size() < n)
      throw std::runtime_error("out of KV blocks: need " + std::to_string(n) + ", free " + std::to_string(free_.size()));
    std::vector<int32_t> got(free_.end() - n, free_.end());
    std::reverse(got.begin(), got.end());
    free_.resize(free_.size() - n);
    o.insert(o.end(), got.begin(), got.end());
    return got;
  }
  int64_t release(int64_t slot) {
    auto& o = at(slot);
    const int64_t n = (int64_t)o.size();
    free_.insert(free_.end(), o.rbegin(), o.rend());
    o.clear();
    return n;
  }
  int64_t truncate(int64_t slot, int64_t n_keep) {
    auto& o = at(slot);
    if (n_keep >= (int64_t)o.size()) return 0;
    const int64_t n = (int64_t)o.size() - n_keep;
    free_.insert(free_.end(), o.rbegin(), o.rbegin() + n);
    o.resize(n_keep);
    return n;
  }

 private:
  std::vector<int32_t>& at(int64_t s) {
    if (s < 0 || s >= (int64_t)owned_.size()) throw std::out_of_range("slot " + std::to_string(s));
    return owned_[s];
  }
  const std::vector<int32_t>& at(int64_t s) const {
    if (s < 0 || s >= (int64_t)owned_.size()) throw std::out_of_range("slot " + std::to_string(s));
    return owned_[s];
  }
  int64_t n_blocks_;
  std::vector<int32_t> free_;
  std::vector<std::vector<int32_t>> owned_;
};

// ------------------------------------------------------------------------------------------ quantization
constexpr int kGroup = 128;

inline int qmax(int bits) { return (1 << (bits - 1)) - 1; }
inline int64_t packed_bytes(int64_t n, int bits) { return bits == 8 ? n : (n * bits + 7) / 8; }

// codes: signed values in [-qmax, qmax], stored offset by qmax in `bits` bits, little-endian bit order
void pack_codes(const int32_t* c, int64_t n, int bits, uint8_t* out) {
  if (bits == 8) {
    for (int64_t i = 0; i < n; ++i) out[i] = (uint8_t)(int8_t)c[i];
    return;
  }
  std::memset(out, 0, packed_bytes(n, bits));
  const int off = qmax(bits);
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t v = (uint32_t)(c[i] + off);
    const int64_t bit = i * bits;
    out[bit >> 3] |= (uint8_t)(v << (bit & 7));
    if ((bit & 7) + bits > 8) out[(bit >> 3) + 1] |= (uint8_t)(v >> (8 - (bit & 7)));
  }
}

inline int32_t unpack_one(const uint8_t* p, int64_t i, int bits) {
  if (bits == 8) return (int8_t)p[i];
  const int64_t bit = i * bits;
  uint32_t w = p[bit >> 3];
  if ((bit & 7) + bits > 8) w |= (uint32_t)p[(bit >> 3) + 1] << 8;
  return (int32_t)((w >> (bit & 7)) & ((1u << bits) - 1)) - qmax(bits);
}

// q = round(x / s), s = absmax / qmax per group of 128 (s = 0 for an all-zero group)
void quantize(const float* x, int64_t n, int bits, uint8_t* codes, float* scales) {
  const int Q = qmax(bits);
  std::vector<int32_t> c(kGroup);
  for (int64_t g = 0; g * kGroup < n; ++g) {
    const int64_t a = g * kGroup, m = std::min<int64_t>(kGroup, n - a);
    float amax = 0.f;
    for (int64_t i = 0; i < m; ++i) amax = std::max(amax, std::fabs(x[a + i]));
    const float s = amax / (float)Q;
    scales[g] = s;
    const float inv = s > 0.f ? 1.f / s : 0.f;
    for (int64_t i = 0; i < m; ++i) c[i] = std::max(-Q, std::min(Q, (int32_t)std::nearbyint(x[a + i] * inv)));
    if (bits == 8) {
      pack_codes(c.data(), m, 8, codes + a);
    } else {
      // groups are packed back to back; 128 codes of 5/6 bits fill whole bytes
      pack_codes(c.data(), m, bits, codes + packed_bytes(a, bits));
    }
  }
}

void dequantize(const uint8_t* codes, const float* scales, int64_t n, int bits, float* x) {
  for (int64_t g = 0; g * kGroup < n; ++g) {
    const int64_t a = g * kGroup, m = std::min<int64_t>(kGroup, n - a);
    const uint8_t* p = bits == 8 ? codes + a : codes + packed_bytes(a, bits);
    for (int64_t i = 0; i < m; ++i) x[a + i] = (float)unpack_one(p, i, bits) * scales[g];
  }
}

std::tuple<torch::Tensor, torch::Tensor> quantize_groups(torch::Tensor x, int64_t bits) {
  TORCH_CHECK(!x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous(), "x: contiguous CPU fp32");
  TORCH_CHECK(bits == 8 || bits == 6 || bits == 5, "bits must be 8, 6 or 5");
  const int64_t n = x.numel();
  auto codes = torch::empty({packed_bytes(n, bits)}, torch::kUInt8);
  auto scales = torch::empty({(n + kGroup - 1) / kGroup}, torch::kFloat);
  quantize(x.data_ptr<float>(), n, bits, codes.data_ptr<uint8_t>(), scales.data_ptr<float>());
  return {codes, scales};
}

torch::Tensor dequantize_groups(torch::Tensor codes, torch::Tensor scales, int64_t n, int64_t bits) {
  TORCH_CHECK(codes.numel() >= packed_bytes(n, bits) && scales.numel() >= (n + kGroup - 1) / kGroup, "sizes");
  auto x = torch::empty({n}, torch::kFloat);
  dequantize(codes.data_ptr<uint8_t>(), scales.data_ptr<float>(), n, bits, x.data_ptr<float>());
  return x;
}

// ------------------------------------------------------------------------------------------ reducer
class HostReducer {
 public:
  explicit HostReducer(int64_t threads) : threads_(std::max<int64_t>(1, threads)) {}

  // contributions: list of (codes, scales) of W ranks, each n elements at `bits`; returns (codes, scales) of
  // the sum requantized to `out_bits`, plus the fp32 sum.
  std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> reduce(std::vector<torch::Tensor> codes,
                                                                std::vector<torch::Tensor> scales, int64_t n,
                                                                int64_t bits, int64_t out_bits) {
    const int64_t W = codes.size();
    TORCH_CHECK(W > 0 && (int64_t)scales.size() == W, "one (codes, scales) pair per rank");
    const int64_t G = (n + kGroup - 1) / kGroup;
    auto sum = torch::zeros({n}, torch::kFloat);
    float* out = sum.data_ptr<float>();
    std::vector<const uint8_t*> cp(W);
    std::vector<const float*> sp(W);
    for (int64_t r = 0; r < W; ++r) {
      TORCH_CHECK(codes[r].numel() >= packed_bytes(n, bits) && scales[r].numel() >= G, "rank ", r, " too short");
      cp[r] = codes[r].data_ptr<uint8_t>();
      sp[r] = scales[r].data_ptr<float>();
    }
    std::atomic<int64_t> next{0};
    auto work = [&]() {
      float tmp[kGroup];
      for (;;) {
        const int64_t g = next.fetch_add(1);
        if (g >= G) return;
        const int64_t a = g * kGroup, m = std::min<int64_t>(kGroup, n - a);
        for (int64_t i = 0; i < m; ++i) tmp[i] = 0.f;
        for (int64_t r = 0; r < W; ++r) {  // fixed rank order: deterministic
          const uint8_t* p = bits == 8 ? cp[r] + a : cp[r] + packed_bytes(a, bits);
          const float s = sp[r][g];
          for (int64_t i = 0; i < m; ++i) {
            const float v = (float)unpack_one(p, i, bits) * s;
            tmp[i] = tmp[i] + v;
          }
        }
        std::memcpy(out + a, tmp, m * sizeof(float));
      }
    };
    std::vector<std::thread> th;
    for (int64_t t = 1; t < threads_; ++t) th.emplace_back(work);
    work();
    for (auto& t : th) t.join();
    auto [oc, os] = quantize_groups(sum, out_bits);
    return {oc, os, sum};
  }

 private:
  int64_t threads_;
};

// ------------------------------------------------------------------------------------------ step log
class StepLog {
 public:
  StepLog(const std::string& path, int64_t n_fields) : n_(n_fields) {
    f_ = std::fopen(path.c_str(), "ab");
    if (!f_) throw std::runtime_error("cannot open " + path);
    std::fseek(f_, 0, SEEK_END);
    if (std::ftell(f_) == 0) {
      const int64_t hdr[2] = {0x474f4c50455453LL /* "STEPLOG" */, n_fields};
      std::fwrite(hdr, sizeof(int64_t), 2, f_);
    }
    buf_.reserve(4096);
  }
  ~StepLog() { close(); }
  void append(const std::vector<int64_t>& rec) {
    if (!f_) throw std::runtime_error("step log closed");
    if ((int64_t)rec.size() != n_) throw std::invalid_argument("record has the wrong field count");
    buf_.insert(buf_.end(), rec.begin(), rec.end());
    if (buf_.size() >= 4096) flush();
  }
  void flush() {
    if (f_ && !buf_.empty()) {
      std::fwrite(buf_.data(), sizeof(int64_t), buf_.size(), f_);
      std::fflush(f_);
      buf_.clear();
    }
  }
  void close() {
    flush();
    if (f_) std::fclose(f_);
    f_ = nullptr;
  }

 private:
  int64_t n_;
  std::FILE* f_ = nullptr;
  std::vector<int64_t> buf_;
};

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "host runtime of arcagi2_flashnext_dots3_b200";
  py::class_<BlockAllocator>(m, "BlockAllocator")
      .def(py::init<int64_t, int64_t>())
      .def("n_free", &BlockAllocator::n_free)
      .def("n_blocks_of", &BlockAllocator::n_blocks_of)
      .def("blocks_of", &BlockAllocator::blocks_of)
      .def("allocate", &BlockAllocator::allocate)
      .def("release", &BlockAllocator::release)
      .def("truncate", &BlockAllocator::truncate);
  m.def("quantize_groups", &quantize_groups);
  m.def("dequantize_groups", &dequantize_groups);
  py::class_<HostReducer>(m, "HostReducer")
      .def(py::init<int64_t>())
      .def("reduce", &HostReducer::reduce, py::call_guard<py::gil_scoped_release>());
  py::class_<StepLog>(m, "StepLog")
      .def(py::init<const std::string&, int64_t>())
      .def("append", &StepLog::append)
      .def("flush", &StepLog::flush)
      .def("close", &StepLog::close);
}
