// loader.cu — safetensors straight to device memory: the reads of
// Model::load (model/model.rs:42, 251-254) through Weights::open / read
// (model/weights.rs:35-81) and Device::upload (model/device.rs:18), fused.
//
// The reference reads each tensor into a Vec<u8>, converts it to a Vec<u16>
// and hands that to `upload`, which copies it to the device: three passes
// over every byte on one thread. Here the header is parsed once and the
// tensor bytes go file -> pinned staging buffer -> GPU with no conversion
// (safetensors stores bf16 little-endian, the device's own layout): worker
// threads each read pieces of up to kPiece bytes with pread into one of two
// pinned buffers and copy them on their own stream, so reading the next
// piece overlaps the copy of the last one. The pinned buffers belong to the
// device and are reused by later loads.
//
// Host only: nothing here launches a kernel.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "runtime.h"

namespace {

constexpr size_t kPiece = size_t(8) << 20;         // bytes per pread + copy (and per staging buffer)
constexpr uint64_t kMaxHeader = uint64_t(100) << 20;  // a larger header is not a safetensors file
constexpr int kMaxThreads = 16;

struct Entry {
  std::string dtype;
  std::vector<size_t> shape;
  uint64_t start = 0, end = 0;  // data_offsets, relative to the end of the header
};

// Just enough of JSON (RFC 8259) to read a safetensors header: a top-level
// object mapping tensor names to {"dtype", "shape", "data_offsets"} objects,
// and "__metadata__", whose value (and any unknown field) is skipped.
class HeaderParser {
 public:
  HeaderParser(const char* p, size_t n) : b_(p), p_(p), e_(p + n) {}

  bool parse(std::unordered_map<std::string, Entry>& out) {
    if (!lit('{')) return bad("the header is not a JSON object");
    if (lit('}')) return end();
    for (;;) {
      std::string name;
      if (!string(name) || !lit(':')) return bad("expected \"name\":");
      if (name == "__metadata__") {
        if (!skip(0)) return false;
      } else {
        Entry e;
        if (!entry(name, e)) return false;
        out[name] = std::move(e);
      }
      if (lit(',')) continue;
      if (lit('}')) return end();
      return bad("expected ',' or '}' in the header object");
    }
  }

  const std::string& error() const { return err_; }

 private:
  const char* b_;
  const char* p_;
  const char* e_;
  std::string err_;

  bool bad(const std::string& m) {
    if (err_.empty()) err_ = m + " (header byte " + std::to_string(consumed()) + ")";
    return false;
  }
  size_t consumed() const { return size_t(p_ - b_); }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(char c) {
    ws();
    if (p_ < e_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  bool end() {
    ws();  // safetensors pads the header with spaces
    return p_ == e_ ? true : bad("bytes after the header object");
  }

  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s += char(cp);
    } else if (cp < 0x800) {
      s += char(0xC0 | (cp >> 6));
      s += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += char(0xE0 | (cp >> 12));
      s += char(0x80 | ((cp >> 6) & 0x3F));
      s += char(0x80 | (cp & 0x3F));
    } else {
      s += char(0xF0 | (cp >> 18));
      s += char(0x80 | ((cp >> 12) & 0x3F));
      s += char(0x80 | ((cp >> 6) & 0x3F));
      s += char(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t& v) {
    if (e_ - p_ < 4) return bad("short \\u escape");
    v = 0;
    for (int i = 0; i < 4; i++) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
      else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
      else return bad("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& s) {
    if (!lit('"')) return bad("expected a string");
    for (;;) {
      if (p_ >= e_) return bad("unterminated string");
      const char c = *p_++;
      if (c == '"') return true;
      if (static_cast<unsigned char>(c) < 0x20) return bad("control character in a string");
      if (c != '\\') {
        s += c;
        continue;
      }
      if (p_ >= e_) return bad("unterminated escape");
      switch (*p_++) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // a high surrogate takes the low one that follows
            uint32_t lo = 0;
            if (e_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return bad("unpaired surrogate");
            p_ += 2;
            if (!hex4(lo)) return false;
            if (lo < 0xDC00 || lo >= 0xE000) return bad("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return bad("unpaired surrogate");
          }
          put_utf8(s, cp);
          break;
        }
        default: return bad("bad escape");
      }
    }
  }
  // A non-negative integer (shapes and offsets): digits only, no overflow.
  bool uint(uint64_t& v) {
    ws();
    if (p_ >= e_ || *p_ < '0' || *p_ > '9') return bad("expected a non-negative integer");
    if (*p_ == '0' && p_ + 1 < e_ && p_[1] >= '0' && p_[1] <= '9') return bad("leading zero");
    v = 0;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
      const uint64_t d = uint64_t(*p_++ - '0');
      if (v > (UINT64_MAX - d) / 10) return bad("integer out of range");
      v = v * 10 + d;
    }
    if (p_ < e_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) return bad("expected an integer");
    return true;
  }
  bool uints(std::vector<uint64_t>& v) {
    if (!lit('[')) return bad("expected an array");
    if (lit(']')) return true;
    for (;;) {
      uint64_t x;
      if (!uint(x)) return false;
      v.push_back(x);
      if (lit(',')) continue;
      if (lit(']')) return true;
      return bad("expected ',' or ']'");
    }
  }
  bool number() {  // any JSON number, skipped
    ws();
    if (p_ < e_ && *p_ == '-') ++p_;
    if (p_ >= e_ || *p_ < '0' || *p_ > '9') return bad("bad number");
    if (*p_ == '0') ++p_;
    else
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    if (p_ < e_ && *p_ == '.') {
      ++p_;
      if (p_ >= e_ || *p_ < '0' || *p_ > '9') return bad("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
      ++p_;
      if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= e_ || *p_ < '0' || *p_ > '9') return bad("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    return true;
  }
  bool word(const char* w) {
    const size_t n = std::strlen(w);
    if (size_t(e_ - p_) < n || std::memcmp(p_, w, n) != 0) return bad("bad literal");
    p_ += n;
    return true;
  }
  bool skip(int depth) {  // any JSON value
    if (depth > 64) return bad("nesting too deep");
    ws();
    if (p_ >= e_) return bad("expected a value");
    switch (*p_) {
      case '"': {
        std::string s;
        return string(s);
      }
      case '{':
        ++p_;
        if (lit('}')) return true;
        for (;;) {
          std::string k;
          if (!string(k) || !lit(':') || !skip(depth + 1)) return bad("bad object");
          if (lit(',')) continue;
          if (lit('}')) return true;
          return bad("expected ',' or '}'");
        }
      case '[':
        ++p_;
        if (lit(']')) return true;
        for (;;) {
          if (!skip(depth + 1)) return false;
          if (lit(',')) continue;
          if (lit(']')) return true;
          return bad("expected ',' or ']'");
        }
      case 't': return word("true");
      case 'f': return word("false");
      case 'n': return word("null");
      default: return number();
    }
  }
  // {"dtype": "...", "shape": [...], "data_offsets": [a, b]}, fields in any
  // order, unknown ones skipped; the three are required (serde's derive).
  bool entry(const std::string& name, Entry& e) {
    if (!lit('{')) return bad("tensor '" + name + "': expected an object");
    bool has_dtype = false, has_shape = false, has_off = false;
    if (!lit('}'))
      for (;;) {
        std::string k;
        if (!string(k) || !lit(':')) return bad("tensor '" + name + "': expected \"field\":");
        if (k == "dtype") {
          e.dtype.clear();
          if (!string(e.dtype)) return false;
          has_dtype = true;
        } else if (k == "shape") {
          std::vector<uint64_t> v;
          if (!uints(v)) return false;
          e.shape.assign(v.begin(), v.end());
          has_shape = true;
        } else if (k == "data_offsets") {
          std::vector<uint64_t> v;
          if (!uints(v)) return false;
          if (v.size() != 2) return bad("tensor '" + name + "': data_offsets needs two integers");
          e.start = v[0];
          e.end = v[1];
          has_off = true;
        } else if (!skip(0)) {
          return false;
        }
        if (lit(',')) continue;
        if (lit('}')) break;
        return bad("tensor '" + name + "': expected ',' or '}'");
      }
    if (!has_dtype) return bad("tensor '" + name + "': missing field `dtype`");
    if (!has_shape) return bad("tensor '" + name + "': missing field `shape`");
    if (!has_off) return bad("tensor '" + name + "': missing field `data_offsets`");
    return true;
  }
};

// An open safetensors file: its descriptor, size, data start and entries.
struct File {
  int fd = -1;
  uint64_t size = 0, data_start = 0;
  std::unordered_map<std::string, Entry> entries;
  ~File() {
    if (fd >= 0) close(fd);
  }
};

// Reads exactly `n` bytes at `off` (read_exact: a short file is an error).
bool read_at(int fd, void* dst, size_t n, uint64_t off, std::string& err) {
  auto* p = static_cast<unsigned char*>(dst);
  while (n > 0) {
    const ssize_t r = pread(fd, p, n, off_t(off));
    if (r < 0) {
      if (errno == EINTR) continue;
      err = std::string("read failed: ") + std::strerror(errno);
      return false;
    }
    if (r == 0) {
      err = "failed to fill whole buffer (unexpected end of file)";
      return false;
    }
    p += r;
    n -= size_t(r);
    off += uint64_t(r);
  }
  return true;
}

// Weights::open (model/weights.rs:35-57): the 8-byte little-endian header
// length, then the JSON header.
int open_file(const char* path, File& f) {
  if (!path) return rt::fail(TB200_ERR_ARG, "null path");
  f.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f.fd < 0) return rt::fail(TB200_ERR_IO, std::string(path) + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(f.fd, &st) != 0) return rt::fail(TB200_ERR_IO, std::string(path) + ": " + std::strerror(errno));
  f.size = uint64_t(st.st_size);
  unsigned char len8[8];
  std::string err;
  if (!read_at(f.fd, len8, 8, 0, err)) return rt::fail(TB200_ERR_IO, std::string(path) + ": " + err);
  uint64_t len = 0;
  for (int i = 7; i >= 0; i--) len = (len << 8) | len8[i];
  if (len > kMaxHeader || 8 + len > f.size)
    return rt::fail(TB200_ERR_FORMAT, std::string(path) + ": header length " + std::to_string(len) +
                                          " does not fit a file of " + std::to_string(f.size) + " bytes");
  std::vector<char> header(len);
  if (!read_at(f.fd, header.data(), len, 8, err)) return rt::fail(TB200_ERR_IO, std::string(path) + ": " + err);
  HeaderParser hp(header.data(), header.size());
  if (!hp.parse(f.entries)) return rt::fail(TB200_ERR_FORMAT, std::string(path) + ": " + hp.error());
  f.data_start = 8 + len;
  return TB200_OK;
}

// Weights::read's checks (model/weights.rs:61-81) plus the ones its
// read_exact and Tensor's length imply: BF16, offsets ordered and inside the
// file, and exactly two bytes per element of the shape.
int check_bf16(const File& f, const std::string& name, const Entry& e, size_t* numel) {
  if (e.dtype != "BF16") return rt::fail(TB200_ERR_FORMAT, "tensor '" + name + "' is " + e.dtype + ", expected BF16");
  size_t n = 1;
  for (size_t s : e.shape) {
    if (s != 0 && n > SIZE_MAX / 2 / s) return rt::fail(TB200_ERR_FORMAT, "tensor '" + name + "': shape too large");
    n *= s;
  }
  if (e.end < e.start || e.end > f.size - f.data_start)
    return rt::fail(TB200_ERR_FORMAT, "tensor '" + name + "': data_offsets [" + std::to_string(e.start) + ", " +
                                          std::to_string(e.end) + "] outside the " +
                                          std::to_string(f.size - f.data_start) + " data bytes");
  if (e.end - e.start != uint64_t(n) * 2)
    return rt::fail(TB200_ERR_FORMAT, "tensor '" + name + "': " + std::to_string(e.end - e.start) +
                                          " bytes for " + std::to_string(n) + " bf16 elements");
  *numel = n;
  return TB200_OK;
}

// One read into a staging buffer and the copy out of it: `len` bytes at
// `file_off`, to `dst` whole (rows == 0) or, for a column window, `rows`
// rows of `width` bytes taken at `src_off` + r * `pitch` of the staged bytes
// and packed at dst + r * width.
struct Piece {
  uint64_t file_off;
  unsigned char* dst;
  size_t len;
  size_t rows = 0, src_off = 0, pitch = 0, width = 0;
};

}  // namespace

int tb200_weight_shape(const tb200_weight* w, size_t* shape, size_t max_ndim, size_t* ndim) {
  ARG_CHECK(w && ndim && (shape || max_ndim == 0), "null argument");
  ARG_CHECK(w->shape.size() <= max_ndim, "the weight has " + std::to_string(w->shape.size()) +
                                             " dimensions, more than max_ndim");
  std::copy(w->shape.begin(), w->shape.end(), shape);
  *ndim = w->shape.size();
  return TB200_OK;
}

int tb200_safetensors_entry(const char* path, const char* name, int* found, char* dtype, size_t dtype_cap,
                            size_t* shape, size_t max_ndim, size_t* ndim, uint64_t* offset, uint64_t* bytes) {
  ARG_CHECK(name && found && ndim && offset && bytes && (shape || max_ndim == 0) && (dtype || dtype_cap == 0),
            "null argument");
  File f;
  if (int rc = open_file(path, f)) return rc;
  const auto it = f.entries.find(name);
  *found = it != f.entries.end();
  if (!*found) return TB200_OK;
  const Entry& e = it->second;
  ARG_CHECK(e.shape.size() <= max_ndim, "tensor '" + std::string(name) + "' has " + std::to_string(e.shape.size()) +
                                            " dimensions, more than max_ndim");
  ARG_CHECK(e.dtype.size() < dtype_cap, "dtype buffer too small");
  std::memcpy(dtype, e.dtype.c_str(), e.dtype.size() + 1);
  std::copy(e.shape.begin(), e.shape.end(), shape);
  *ndim = e.shape.size();
  *offset = f.data_start + e.start;
  *bytes = e.end >= e.start ? e.end - e.start : 0;
  return TB200_OK;
}

namespace {

// tb200_upload_safetensors with optional windows (null: every tensor whole).
int upload_impl(tb200_device* d, const char* path, const char* const* names, const tb200_window* win, size_t n,
                int threads, tb200_weight** out) {
  if (int rc = rt::use(d)) return rc;
  ARG_CHECK(out && (names || n == 0), "null argument");
  ARG_CHECK(threads >= 0 && threads <= kMaxThreads, "threads must be 0 (automatic) .. " + std::to_string(kMaxThreads));
  for (size_t i = 0; i < n; i++) out[i] = nullptr;
  for (size_t i = 0; i < n; i++) ARG_CHECK(names[i], "null tensor name");
  File f;
  if (int rc = open_file(path, f)) return rc;

  // Check every requested tensor before allocating anything.
  std::vector<size_t> numel(n, 0);
  std::vector<const Entry*> ent(n, nullptr);
  for (size_t i = 0; i < n; i++) {
    const auto it = f.entries.find(names[i]);
    if (it == f.entries.end()) continue;  // Weights::contains is false: the caller decides
    ent[i] = &it->second;
    if (int rc = check_bf16(f, it->first, it->second, &numel[i])) return rc;
    if (!win || (win[i].rows == 0 && win[i].cols == 0)) continue;
    const tb200_window& wi = win[i];
    const std::vector<size_t>& sh = it->second.shape;
    const std::string nm = "tensor '" + it->first + "': ";
    ARG_CHECK(sh.size() == 2, nm + "a window needs a matrix");
    ARG_CHECK(wi.rows > 0 && wi.cols > 0, nm + "an empty window");
    ARG_CHECK(wi.row0 <= sh[0] && wi.rows <= sh[0] - wi.row0 && wi.col0 <= sh[1] && wi.cols <= sh[1] - wi.col0,
              nm + "window rows " + std::to_string(wi.row0) + "+" + std::to_string(wi.rows) + ", columns " +
                  std::to_string(wi.col0) + "+" + std::to_string(wi.cols) + " outside its " + std::to_string(sh[0]) +
                  " x " + std::to_string(sh[1]));
    ARG_CHECK(wi.cols == sh[1] || sh[1] * 2 <= kPiece,
              nm + "rows wider than " + std::to_string(kPiece / 2) + " elements take no column window");
    numel[i] = wi.rows * wi.cols;
  }

  std::vector<tb200_weight*> made;
  auto undo = [&](int rc) {  // every worker has finished (and synchronized its stream)
    for (tb200_weight* w : made) {
      cudaFree(w->ptr);
      delete w;
    }
    for (size_t i = 0; i < n; i++) out[i] = nullptr;
    return rc;
  };
  std::vector<Piece> pieces;
  for (size_t i = 0; i < n; i++) {
    if (!ent[i]) continue;
    auto* w = new tb200_weight;
    const bool whole = !win || (win[i].rows == 0 && win[i].cols == 0);
    w->shape = whole ? ent[i]->shape : std::vector<size_t>{win[i].rows, win[i].cols};
    w->numel = numel[i];
    made.push_back(w);
    out[i] = w;
    if (!w->numel) continue;
    const cudaError_t e = cudaMalloc(&w->ptr, w->numel * 2);
    if (e != cudaSuccess) {
      w->ptr = nullptr;
      return undo(rt::fail(TB200_ERR_CUDA, std::string("upload_safetensors: ") + cudaGetErrorString(e)));
    }
    unsigned char* dst = reinterpret_cast<unsigned char*>(w->ptr);
    uint64_t base = f.data_start + ent[i]->start;
    if (!whole && win[i].cols == ent[i]->shape[1]) {  // whole rows: one contiguous run
      base += uint64_t(win[i].row0) * win[i].cols * 2;
    } else if (!whole) {  // a column window: stage whole rows, copy their middle out
      const size_t pitch = ent[i]->shape[1] * 2, width = win[i].cols * 2;
      const size_t per = std::max<size_t>(1, kPiece / pitch);  // rows per piece
      for (size_t r = 0; r < win[i].rows; r += per) {
        const size_t nr = std::min(per, win[i].rows - r);
        Piece pc{base + uint64_t(win[i].row0 + r) * pitch, dst + r * width, nr * pitch};
        pc.rows = nr;
        pc.src_off = win[i].col0 * 2;
        pc.pitch = pitch;
        pc.width = width;
        pieces.push_back(pc);
      }
      continue;
    }
    for (size_t off = 0; off < w->numel * 2; off += kPiece)
      pieces.push_back({base + off, dst + off, std::min(kPiece, w->numel * 2 - off)});
  }
  if (pieces.empty()) return TB200_OK;

  int nt = threads ? threads : int(std::min(8u, std::max(1u, std::thread::hardware_concurrency())));
  nt = int(std::min<size_t>(size_t(nt), pieces.size()));
  while (d->stage.size() < size_t(2 * nt)) {
    void* p = nullptr;
    const cudaError_t e = cudaHostAlloc(&p, kPiece, cudaHostAllocDefault);
    if (e != cudaSuccess)
      return undo(rt::fail(TB200_ERR_CUDA, std::string("upload_safetensors: pinned staging: ") + cudaGetErrorString(e)));
    d->stage.push_back(p);
  }
  std::atomic<size_t> next{0};
  std::atomic<bool> failed{false};
  std::mutex mu;
  std::string first_err;
  int first_code = TB200_OK;
  auto record = [&](int code, const std::string& m) {
    std::lock_guard<std::mutex> g(mu);
    if (first_code == TB200_OK) {
      first_code = code;
      first_err = m;
    }
    failed = true;
  };
  const int ordinal = d->ordinal;
  auto worker = [&](int t) {
    cudaStream_t s = nullptr;
    void* buf[2] = {d->stage[size_t(2 * t)], d->stage[size_t(2 * t + 1)]};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};
    cudaError_t e = cudaSetDevice(ordinal);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && e == cudaSuccess; b++) e = cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming);
    if (e != cudaSuccess) record(TB200_ERR_CUDA, std::string("upload_safetensors: ") + cudaGetErrorString(e));
    for (unsigned k = 0; e == cudaSuccess && !failed; k++) {
      const size_t i = next.fetch_add(1);
      if (i >= pieces.size()) break;
      const int b = int(k & 1);
      if (pending[b]) {  // this buffer's last copy has left it
        e = cudaEventSynchronize(ev[b]);
        if (e != cudaSuccess) break;
      }
      std::string err;
      if (!read_at(f.fd, buf[b], pieces[i].len, pieces[i].file_off, err)) {
        record(TB200_ERR_IO, std::string(path) + ": " + err);
        break;
      }
      const Piece& pc = pieces[i];
      e = pc.rows ? cudaMemcpy2DAsync(pc.dst, pc.width, static_cast<unsigned char*>(buf[b]) + pc.src_off, pc.pitch,
                                      pc.width, pc.rows, cudaMemcpyHostToDevice, s)
                  : cudaMemcpyAsync(pc.dst, buf[b], pc.len, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess) e = cudaEventRecord(ev[b], s);
      pending[b] = true;
    }
    if (s) {
      const cudaError_t e2 = cudaStreamSynchronize(s);
      if (e == cudaSuccess) e = e2;
    }
    if (e != cudaSuccess) record(TB200_ERR_CUDA, std::string("upload_safetensors: ") + cudaGetErrorString(e));
    for (int b = 0; b < 2; b++)
      if (ev[b]) cudaEventDestroy(ev[b]);
    if (s) cudaStreamDestroy(s);
  };
  std::vector<std::thread> pool;
  pool.reserve(size_t(nt));
  for (int t = 0; t < nt; t++) {
    try {
      pool.emplace_back(worker, t);
    } catch (const std::exception& ex) {  // no thread: stop the others, report (nothing crosses the C ABI)
      record(TB200_ERR_IO, std::string("upload_safetensors: cannot start a worker thread: ") + ex.what());
      break;
    }
  }
  for (auto& t : pool) t.join();
  if (first_code != TB200_OK) return undo(rt::fail(first_code, first_err));
  return TB200_OK;
}

}  // namespace

int tb200_upload_safetensors(tb200_device* d, const char* path, const char* const* names, size_t n, int threads,
                             tb200_weight** out) {
  return upload_impl(d, path, names, nullptr, n, threads, out);
}

int tb200_upload_safetensors_windows(tb200_device* d, const char* path, const char* const* names,
                                     const tb200_window* windows, size_t n, int threads, tb200_weight** out) {
  if (!windows && n) {
    if (out)
      for (size_t i = 0; i < n; i++) out[i] = nullptr;
    return rt::fail(TB200_ERR_ARG, "null windows");
  }
  return upload_impl(d, path, names, windows, n, threads, out);
}
