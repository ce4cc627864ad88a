// nq8_host.cpp -- host-side weight preparation for libnq8.so:
//   * repack GGUF Q8_0 blocks into the tiled HBM layout (and back),
//   * Q8_0 quantization with ggml semantics (for nq_weight_from_f32),
//   * a bounds-checked GGUF v2/v3 reader over mmap.
#include "nq8_host.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace nq {

// Run fn(lo, hi) over [0, n) on up to the host's hardware threads, in
// contiguous ranges (each index in exactly one range).  Small ranges run
// inline.
template <class Fn>
static void parallel_ranges(int64_t n, int64_t min_per_thread, Fn fn) {
  const int64_t hw = std::max(1u, std::thread::hardware_concurrency());
  const int64_t parts = std::min<int64_t>(hw, std::max<int64_t>(1, n / std::max<int64_t>(1, min_per_thread)));
  if (parts <= 1) {
    fn(int64_t{0}, n);
    return;
  }
  std::vector<std::thread> th;
  const int64_t step = (n + parts - 1) / parts;
  for (int64_t lo = 0; lo < n; lo += step) th.emplace_back(fn, lo, std::min(n, lo + step));
  for (auto &t : th) t.join();
}

// ------------------------------------------------------------------ layout
int pack_n_tiles(int64_t n, int flags) {
  if (flags & kPackGlu) return static_cast<int>((n / 2 + 63) / 64);
  return static_cast<int>((n + kPackRows - 1) / kPackRows);
}
int pack_k_chunks(int64_t k) { return static_cast<int>((k + kPackK - 1) / kPackK); }

// Source row of local row r of tile t, or -1 for a zero padding row.
static int64_t src_row(int64_t n, int flags, int t, int r) {
  if (flags & kPackGlu) {
    const int64_t half = n / 2;
    const int64_t v = static_cast<int64_t>(t) * 64 + (r & 63);
    if (v >= half) return -1;
    return r < 64 ? v : half + v;
  }
  const int64_t row = static_cast<int64_t>(t) * kPackRows + r;
  return row < n ? row : -1;
}

void pack_q8_0(const uint8_t *blocks, int64_t n, int64_t k, int flags, uint8_t *out) {
  const int tiles = pack_n_tiles(n, flags);
  const int kc = pack_k_chunks(k);
  const int64_t kb = k / 32;
  std::memset(out, 0, static_cast<size_t>(tiles) * kc * kTileBytes);
  // tiles are independent (each writes its own kc chunks)
  parallel_ranges(tiles, 64, [&](int64_t t0, int64_t t1) {
  for (int t = static_cast<int>(t0); t < t1; ++t)
    for (int r = 0; r < kPackRows; ++r) {
      const int64_t sr = src_row(n, flags, t, r);
      if (sr < 0) continue;
      const uint8_t *srow = blocks + sr * kb * 34;
      for (int c = 0; c < kc; ++c) {
        uint8_t *tile = out + (static_cast<size_t>(t) * kc + c) * kTileBytes;
        for (int h = 0; h < 2; ++h) {
          const int64_t b = static_cast<int64_t>(c) * 2 + h;
          if (b >= kb) continue;
          const uint8_t *blk = srow + b * 34;
          std::memcpy(tile + qs_offset(r, 2 * h), blk + 2, 16);
          std::memcpy(tile + qs_offset(r, 2 * h + 1), blk + 2 + 16, 16);
          std::memcpy(tile + scale_offset(r, h), blk, 2);
        }
      }
    }
  });
}

static uint16_t f32_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return static_cast<uint16_t>(x >> 16);
}

void pack_bf16_rows(const float *w, int64_t n, int64_t k, int flags, uint16_t *out) {
  const int tiles = pack_n_tiles(n, flags);
  const int64_t k_pad = static_cast<int64_t>(pack_k_chunks(k)) * kPackK;
  for (int t = 0; t < tiles; ++t)
    for (int r = 0; r < kPackRows; ++r) {
      uint16_t *dst = out + (static_cast<int64_t>(t) * kPackRows + r) * k_pad;
      const int64_t sr = src_row(n, flags, t, r);
      for (int64_t c = 0; c < k_pad; ++c) dst[c] = (sr >= 0 && c < k) ? f32_to_bf16(w[sr * k + c]) : 0;
    }
}

void unpack_q8_0(const uint8_t *packed, int64_t n, int64_t k, int flags, uint8_t *blocks) {
  const int tiles = pack_n_tiles(n, flags);
  const int kc = pack_k_chunks(k);
  const int64_t kb = k / 32;
  for (int t = 0; t < tiles; ++t)
    for (int r = 0; r < kPackRows; ++r) {
      const int64_t sr = src_row(n, flags, t, r);
      if (sr < 0) continue;
      uint8_t *drow = blocks + sr * kb * 34;
      for (int c = 0; c < kc; ++c) {
        const uint8_t *tile = packed + (static_cast<size_t>(t) * kc + c) * kTileBytes;
        for (int h = 0; h < 2; ++h) {
          const int64_t b = static_cast<int64_t>(c) * 2 + h;
          if (b >= kb) continue;
          uint8_t *blk = drow + b * 34;
          std::memcpy(blk + 2, tile + qs_offset(r, 2 * h), 16);
          std::memcpy(blk + 2 + 16, tile + qs_offset(r, 2 * h + 1), 16);
          std::memcpy(blk, tile + scale_offset(r, h), 2);
        }
      }
    }
}

// --------------------------------------------------------------- quantize
// IEEE binary16, round to nearest even, subnormals, overflow to inf.
static uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t a = x & 0x7fffffffu;
  if (a >= 0x7f800000u) return static_cast<uint16_t>(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (a >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);
  if (a < 0x38800000u) {
    if (a < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t e = a >> 23;
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;
    const uint32_t sh = 126u - e;
    uint32_t r = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u);
    const uint32_t hf = 1u << (sh - 1u);
    if (rem > hf || (rem == hf && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
  }
  uint32_t r = a - 0x38000000u;
  const uint32_t rem = r & 0x1fffu;
  r >>= 13;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return static_cast<uint16_t>(sign | r);
}

// ggml quantize_row_q8_0_ref semantics: d = amax/127, q = roundf(x / d).
static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      int sh = 0;
      while (!(m & 0x400u)) {
        m <<= 1;
        ++sh;
      }
      x = sign | (static_cast<uint32_t>(113 - sh) << 23) | ((m & 0x3ffu) << 13);
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

int64_t q8_0_first_mismatch(const float *w, const uint8_t *blocks, int64_t count) {
  for (int64_t b = 0; b < count / 32; ++b) {
    uint16_t dh;
    std::memcpy(&dh, blocks + b * 34, 2);
    const float d = f16_to_f32(dh);
    for (int j = 0; j < 32; ++j) {
      const float v = d * static_cast<float>(static_cast<int8_t>(blocks[b * 34 + 2 + j]));
      if (!(v == w[b * 32 + j])) return b * 32 + j;
    }
  }
  return -1;
}

void quantize_q8_0(const float *w, int64_t n, int64_t k, uint8_t *blocks) {
  const int64_t nb = n * (k / 32);
  // blocks are independent
  parallel_ranges(nb, 1 << 15, [&](int64_t b0, int64_t b1) {
  for (int64_t b = b0; b < b1; ++b) {
    const float *xb = w + b * 32;
    uint8_t *ob = blocks + b * 34;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    const uint16_t dh = f32_to_f16(d);
    std::memcpy(ob, &dh, 2);
    for (int j = 0; j < 32; ++j) ob[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(std::roundf(xb[j] * id)));
  }
  });
}

// --------------------------------------------------------------------- GGUF
namespace {
struct Reader {
  const uint8_t *p;
  size_t size;
  size_t off;
  bool ok = true;
  template <class T>
  T get() {
    T v{};
    if (off + sizeof(T) > size) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + off, sizeof(T));
    off += sizeof(T);
    return v;
  }
  bool skip(uint64_t n) {
    if (n > size - off) {
      ok = false;
      return false;
    }
    off += n;
    return true;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (!ok || len > size - off) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char *>(p + off), len);
    off += len;
    return s;
  }
};

int scalar_size(uint32_t type) {
  switch (type) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return -1;
  }
}

bool skip_value(Reader &r, uint32_t type, int depth) {
  if (depth > 4) return false;
  if (type == 8) {
    r.str();
    return r.ok;
  }
  if (type == 9) {
    const uint32_t et = r.get<uint32_t>();
    const uint64_t cnt = r.get<uint64_t>();
    if (!r.ok) return false;
    const int es = scalar_size(et);
    if (es > 0) {
      if (cnt > (r.size - r.off) / es) return false;
      return r.skip(cnt * es);
    }
    for (uint64_t i = 0; i < cnt; ++i)
      if (!skip_value(r, et, depth + 1)) return false;
    return true;
  }
  const int s = scalar_size(type);
  return s > 0 && r.skip(s);
}
}  // namespace

GgufFile::~GgufFile() {
  if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
  if (fd_ >= 0) close(fd_);
}

int GgufFile::open(const char *path, std::string *err) {
  fd_ = ::open(path, O_RDONLY);
  if (fd_ < 0) {
    *err = std::string("cannot open ") + path;
    return kErrIo;
  }
  struct stat st;
  if (fstat(fd_, &st) != 0 || st.st_size < 24) {
    *err = "GGUF file too small";
    return kErrFormat;
  }
  size_ = static_cast<size_t>(st.st_size);
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (map_ == MAP_FAILED) {
    *err = "mmap failed";
    return kErrIo;
  }
  Reader r{static_cast<const uint8_t *>(map_), size_, 0};
  const uint32_t magic = r.get<uint32_t>();
  const uint32_t version = r.get<uint32_t>();
  if (magic != 0x46554747u) {
    *err = "not a GGUF file (bad magic)";
    return kErrFormat;
  }
  if (version < 2 || version > 3) {
    *err = "unsupported GGUF version " + std::to_string(version);
    return kErrFormat;
  }
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
    *err = "GGUF header counts out of range";
    return kErrFormat;
  }
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv; ++i) {
    const std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    if (!r.ok) break;
    if (key == "general.alignment" && type == 4) {
      alignment = r.get<uint32_t>();
      continue;
    }
    if (!skip_value(r, type, 0)) {
      r.ok = false;
      break;
    }
  }
  if (!r.ok || alignment == 0 || (alignment & (alignment - 1))) {
    *err = "malformed GGUF key/value section";
    return kErrFormat;
  }
  tensors_.clear();
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd > 4) {
      *err = "malformed GGUF tensor info";
      return kErrFormat;
    }
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (!r.ok) {
      *err = "malformed GGUF tensor info";
      return kErrFormat;
    }
    tensors_.push_back(t);
  }
  data_start_ = (r.off + alignment - 1) / alignment * alignment;
  if (data_start_ > size_) {
    *err = "GGUF data section beyond end of file";
    return kErrFormat;
  }
  return 0;
}

const GgufTensor *GgufFile::find(const char *name) const {
  for (const auto &t : tensors_)
    if (t.name == name) return &t;
  return nullptr;
}

const uint8_t *GgufFile::data(const GgufTensor &t, size_t bytes) const {
  const size_t start = data_start_ + t.offset;
  if (t.offset > size_ || start > size_ || bytes > size_ - start) return nullptr;
  return static_cast<const uint8_t *>(map_) + start;
}

}  // namespace nq
