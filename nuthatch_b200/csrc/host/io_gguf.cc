// TensorSource (positioned reads) and the GGUF metadata parser.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "nuthatch/gguf_file.h"
#include "nuthatch/tensor_source.h"

namespace nuthatch {

// ------------------------------------------------------------ TensorSource
std::unique_ptr<TensorSource> TensorSource::Open(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return nullptr;
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    return nullptr;
  }
  return std::unique_ptr<TensorSource>(new TensorSource(fd, static_cast<size_t>(st.st_size)));
}

TensorSource::~TensorSource() {
  if (fd_ >= 0) ::close(fd_);
}

bool TensorSource::ReadAt(size_t offset, size_t size, void* out) const {
  auto* dst = static_cast<uint8_t*>(out);
  size_t done = 0;
  while (done < size) {
    const ssize_t n = ::pread(fd_, dst + done, size - done, static_cast<off_t>(offset + done));
    if (n <= 0) return false;  // read error, or end of file before `size` bytes
    done += static_cast<size_t>(n);
  }
  return true;
}

// ------------------------------------------------------------ GGUF
size_t RowBytes(int32_t type, int64_t n) {
  if (type == kTypeF32) return static_cast<size_t>(n) * 4;
  if (n % 256 != 0) return 0;
  if (type == kTypeQ4K) return static_cast<size_t>(n / 256) * 144;
  if (type == kTypeQ6K) return static_cast<size_t>(n / 256) * 210;
  return 0;
}

namespace {

// Sequential reader over a file with a small buffer.
class Reader {
 public:
  explicit Reader(const TensorSource& src) : src_(src) {}
  bool Bytes(void* out, size_t n) {
    if (!ok_) return false;
    if (pos_ + n > src_.file_size() || !src_.ReadAt(pos_, n, out)) {
      ok_ = false;
      return false;
    }
    pos_ += n;
    return true;
  }
  template <typename T>
  T Get() {
    T v{};
    Bytes(&v, sizeof(T));
    return v;
  }
  bool Str(std::string* s) {
    const uint64_t n = Get<uint64_t>();
    if (!ok_ || n > (1ull << 30)) return ok_ = false;
    s->resize(n);
    return n == 0 || Bytes(&(*s)[0], n);
  }
  bool Skip(uint32_t type, int depth = 0) {
    static const size_t sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (depth > 4) return ok_ = false;
    if (type == 8) {
      std::string s;
      return Str(&s);
    }
    if (type == 9) {
      const uint32_t et = Get<uint32_t>();
      const uint64_t n = Get<uint64_t>();
      if (!ok_) return false;
      if (et != 8 && et != 9 && et < 13) {
        if (n > (1ull << 40) / (sz[et] ? sz[et] : 1)) return ok_ = false;
        pos_ += n * sz[et];
        if (pos_ > src_.file_size()) return ok_ = false;
        return true;
      }
      for (uint64_t i = 0; i < n && ok_; ++i) Skip(et, depth + 1);
      return ok_;
    }
    if (type >= 13) return ok_ = false;
    pos_ += sz[type];
    if (pos_ > src_.file_size()) return ok_ = false;
    return true;
  }
  bool ok() const { return ok_; }
  uint64_t pos() const { return pos_; }

 private:
  const TensorSource& src_;
  uint64_t pos_ = 0;
  bool ok_ = true;
};

}  // namespace

std::unique_ptr<GgufFile> GgufFile::Open(const std::string& path) {
  auto src = TensorSource::Open(path);
  if (src == nullptr) return nullptr;
  Reader r(*src);
  char magic[4];
  if (!r.Bytes(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return nullptr;
  std::unique_ptr<GgufFile> g(new GgufFile());
  g->version_ = r.Get<uint32_t>();
  if (g->version_ != 2 && g->version_ != 3) return nullptr;
  const uint64_t n_tensors = r.Get<uint64_t>();
  const uint64_t n_kv = r.Get<uint64_t>();
  if (!r.ok() || n_tensors > (1u << 24) || n_kv > (1u << 24)) return nullptr;
  for (uint64_t i = 0; i < n_kv && r.ok(); ++i) {
    std::string key;
    if (!r.Str(&key)) return nullptr;
    const uint32_t type = r.Get<uint32_t>();
    if (type == 4) {
      g->u32_[key] = r.Get<uint32_t>();
    } else if (type == 6) {
      g->f32_[key] = r.Get<float>();
    } else if (type == 8) {
      std::string v;
      if (!r.Str(&v)) return nullptr;
      g->str_[key] = v;
    } else if (!r.Skip(type)) {
      return nullptr;
    }
  }
  uint32_t alignment = 32;
  g->GetU32("general.alignment", &alignment);
  if (alignment == 0 || (alignment & (alignment - 1)) != 0) return nullptr;
  for (uint64_t i = 0; i < n_tensors && r.ok(); ++i) {
    GgufTensorInfo t;
    if (!r.Str(&t.name)) return nullptr;
    t.n_dims = r.Get<uint32_t>();
    if (t.n_dims == 0 || t.n_dims > 4) return nullptr;
    for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = static_cast<int64_t>(r.Get<uint64_t>());
    t.type = static_cast<int32_t>(r.Get<uint32_t>());
    t.offset = r.Get<uint64_t>();
    g->tensors_.push_back(t);
  }
  if (!r.ok()) return nullptr;
  g->data_offset_ = (r.pos() + alignment - 1) / alignment * alignment;
  for (size_t i = 0; i < g->tensors_.size(); ++i) {
    GgufTensorInfo& t = g->tensors_[i];
    for (int d = 0; d < 4; ++d)
      if (t.ne[d] <= 0) return nullptr;
    const size_t rb = RowBytes(t.type, t.ne[0]);
    if (rb == 0) return nullptr;  // unsupported type or a row not a block multiple
    t.nb[0] = t.type == kTypeF32 ? 4 : 0;
    t.nb[1] = rb;
    t.nb[2] = rb * t.ne[1];
    t.nb[3] = t.nb[2] * t.ne[2];
    t.nbytes = t.nb[3] * t.ne[3];
    t.offset += g->data_offset_;
    if (t.offset + t.nbytes > src->file_size()) return nullptr;
    g->index_[t.name] = i;
  }
  return g;
}

bool ReadGgufStringArrays(const std::string& path, const std::vector<std::string>& keys,
                          std::unordered_map<std::string, std::vector<std::string>>* out) {
  out->clear();
  auto src = TensorSource::Open(path);
  if (src == nullptr) return false;
  Reader r(*src);
  char magic[4];
  if (!r.Bytes(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return false;
  const uint32_t version = r.Get<uint32_t>();
  if (version != 2 && version != 3) return false;
  r.Get<uint64_t>();  // tensor count
  const uint64_t n_kv = r.Get<uint64_t>();
  if (!r.ok() || n_kv > (1u << 24)) return false;
  for (uint64_t i = 0; i < n_kv && r.ok(); ++i) {
    std::string key;
    if (!r.Str(&key)) return false;
    const uint32_t type = r.Get<uint32_t>();
    const bool wanted = std::find(keys.begin(), keys.end(), key) != keys.end();
    if (wanted && type == 9) {
      const uint32_t et = r.Get<uint32_t>();
      const uint64_t n = r.Get<uint64_t>();
      // Every string takes at least its 8-byte length: a count beyond what
      // the file holds is corrupt (and must not size an allocation).
      if (!r.ok() || n > (src->file_size() - r.pos()) / 8) return false;
      if (et == 8) {
        std::vector<std::string> v(n);
        for (uint64_t j = 0; j < n; ++j)
          if (!r.Str(&v[j])) return false;
        (*out)[key] = std::move(v);
        continue;
      }
      for (uint64_t j = 0; j < n && r.ok(); ++j) r.Skip(et, 1);
      if (!r.ok()) return false;
      continue;
    }
    if (!r.Skip(type)) return false;
  }
  return r.ok();
}

bool GgufFile::GetU32(const std::string& key, uint32_t* out) const {
  auto it = u32_.find(key);
  if (it == u32_.end()) return false;
  *out = it->second;
  return true;
}
bool GgufFile::GetF32(const std::string& key, float* out) const {
  auto it = f32_.find(key);
  if (it == f32_.end()) return false;
  *out = it->second;
  return true;
}
bool GgufFile::GetStr(const std::string& key, std::string* out) const {
  auto it = str_.find(key);
  if (it == str_.end()) return false;
  *out = it->second;
  return true;
}
const GgufTensorInfo* GgufFile::tensor(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

}  // namespace nuthatch
