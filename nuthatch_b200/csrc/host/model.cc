// OlmoeModel (resident in HBM), KvCache, StreamingModel, ExpertReader.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "nuthatch/expert_reader.h"
#include "nuthatch/gguf_file.h"
#include "nuthatch/kv_cache.h"
#include "nuthatch/olmoe_model.h"
#include "nuthatch/streaming_model.h"
#include "nuthatch/tensor_source.h"
#include "workspace.h"

namespace nuthatch {

namespace {

constexpr size_t kAlignDev = 256;
constexpr size_t kTailPad = 256;
constexpr size_t kChunk = 64ull << 20;

size_t AlignUp(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool IsExpertTensor(const std::string& name) { return name.find("_exps.weight") != std::string::npos; }

// Copies file bytes [off, off+n) to device memory through two pinned bounce buffers.
class Uploader {
 public:
  Uploader() {
    for (int i = 0; i < 2; ++i) {
      if (cudaHostAlloc(&buf_[i], kChunk, cudaHostAllocDefault) != cudaSuccess) buf_[i] = nullptr;
      cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming);
    }
    cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
  }
  ~Uploader() {
    if (stream_) cudaStreamSynchronize(stream_);
    for (int i = 0; i < 2; ++i) {
      if (buf_[i]) cudaFreeHost(buf_[i]);
      if (ev_[i]) cudaEventDestroy(ev_[i]);
    }
    if (stream_) cudaStreamDestroy(stream_);
  }
  bool ok() const { return buf_[0] != nullptr && buf_[1] != nullptr && stream_ != nullptr; }
  bool Copy(const TensorSource& src, uint64_t off, size_t n, uint8_t* dst) {
    size_t done = 0;
    while (done < n) {
      const size_t take = std::min(kChunk, n - done);
      cudaEventSynchronize(ev_[cur_]);  // the previous copy out of this buffer is complete
      if (!src.ReadAt(off + done, take, buf_[cur_])) return false;
      if (cudaMemcpyAsync(dst + done, buf_[cur_], take, cudaMemcpyHostToDevice, stream_) != cudaSuccess) return false;
      cudaEventRecord(ev_[cur_], stream_);
      cur_ ^= 1;
      done += take;
    }
    return true;
  }
  bool Sync() { return cudaStreamSynchronize(stream_) == cudaSuccess; }

 private:
  void* buf_[2] = {nullptr, nullptr};
  cudaEvent_t ev_[2] = {nullptr, nullptr};
  cudaStream_t stream_ = nullptr;
  int cur_ = 0;
};

}  // namespace

OlmoeConfig ParseOlmoeConfig(const GgufFile& g) {
  std::string arch;
  if (!g.GetStr("general.architecture", &arch) || arch.empty()) arch = "olmoe";
  auto U = [&](const char* k, uint32_t def) {
    uint32_t v = def;
    g.GetU32(arch + "." + k, &v);
    return v;
  };
  auto F = [&](const char* k, float def) {
    float v = def;
    g.GetF32(arch + "." + k, &v);
    return v;
  };
  OlmoeConfig c;
  c.n_layers = U("block_count", 0);
  c.n_embd = U("embedding_length", 0);
  c.n_head = U("attention.head_count", 0);
  c.n_head_kv = U("attention.head_count_kv", c.n_head);
  c.n_ff = U("feed_forward_length", 0);
  c.n_expert = U("expert_count", 0);
  c.n_expert_used = U("expert_used_count", 0);
  c.n_ctx_train = U("context_length", 0);
  c.rope_freq_base = F("rope.freq_base", 10000.0f);
  c.rms_eps = F("attention.layer_norm_rms_epsilon", 1e-5f);
  const GgufTensorInfo* out = g.tensor("output.weight");
  if (out == nullptr) out = g.tensor("token_embd.weight");
  if (out != nullptr) c.n_vocab = static_cast<uint32_t>(out->ne[1]);
  return c;
}

namespace {

// Which experts of each expert tensor go to the device: none (streaming),
// all, or a contiguous shard [first, first + count) (expert parallelism).
struct ExpertPick {
  bool skip = false;
  uint32_t first = 0, count = 0;  // count 0: all
};

// Bytes of tensor t that are uploaded, and where they start in the file.
void Slice(const GgufTensorInfo& t, const ExpertPick& pick, uint64_t* offset, size_t* nbytes) {
  *offset = t.offset;
  *nbytes = t.nbytes;
  if (pick.count != 0 && IsExpertTensor(t.name)) {
    *offset = t.offset + static_cast<uint64_t>(pick.first) * t.nb[2];
    *nbytes = static_cast<size_t>(pick.count) * t.nb[2];
  }
}

// Allocates one device region for the selected tensors and uploads them.
bool UploadTensors(const std::string& path, const GgufFile& g, const ExpertPick& pick,
                   std::unordered_map<std::string, DTensor>* out, void** base, size_t* bytes) {
  size_t total = 0;
  std::vector<std::pair<const GgufTensorInfo*, size_t>> plan;
  for (const GgufTensorInfo& t : g.tensors()) {
    if (pick.skip && IsExpertTensor(t.name)) continue;
    if (pick.count != 0 && IsExpertTensor(t.name) && (t.ne[2] < pick.first + pick.count || t.nb[2] == 0))
      return false;
    uint64_t off = 0;
    size_t nb = 0;
    Slice(t, pick, &off, &nb);
    plan.push_back({&t, total});
    total += AlignUp(nb, kAlignDev);
  }
  total += kTailPad;
  void* dev = nullptr;
  if (cudaMalloc(&dev, total) != cudaSuccess) return false;
  // The uploads below run on a non-blocking stream, which does not order
  // itself after the legacy stream: finish the zeroing first.
  if (cudaMemset(dev, 0, total) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(dev);
    return false;
  }
  auto src = TensorSource::Open(path);
  Uploader up;
  bool ok = src != nullptr && up.ok();
  for (auto& pt : plan) {
    if (!ok) break;
    const GgufTensorInfo& t = *pt.first;
    uint8_t* dst = static_cast<uint8_t*>(dev) + pt.second;
    uint64_t off = 0;
    size_t nb = 0;
    Slice(t, pick, &off, &nb);
    ok = up.Copy(*src, off, nb, dst);
    DTensor d;
    d.name = t.name;
    d.type = t.type;
    for (int i = 0; i < 4; ++i) {
      d.ne[i] = t.ne[i];
      d.nb[i] = t.nb[i];
    }
    if (pick.count != 0 && IsExpertTensor(t.name)) d.ne[2] = pick.count;
    d.data = dst;
    d.nbytes = nb;
    (*out)[t.name] = d;
  }
  ok = up.Sync() && ok;
  if (!ok) {
    cudaFree(dev);
    out->clear();
    return false;
  }
  *base = dev;
  *bytes = total;
  return true;
}

}  // namespace

std::unique_ptr<OlmoeModel> OlmoeModel::Load(const std::string& path) {
  auto g = GgufFile::Open(path);
  if (g == nullptr) return nullptr;
  std::unique_ptr<OlmoeModel> m(new OlmoeModel());
  m->cfg_ = ParseOlmoeConfig(*g);
  m->expert_count_ = m->cfg_.n_expert;
  cudaGetDevice(&m->device_);
  if (!UploadTensors(path, *g, ExpertPick{}, &m->tensors_, &m->base_, &m->bytes_)) return nullptr;
  m->ws_.reset(new Workspace(m->cfg_));
  m->ws_->view_ok = BuildView(*m, true, &m->ws_->view);
  return m;
}

std::unique_ptr<OlmoeModel> OlmoeModel::LoadExpertShard(const std::string& path, uint32_t first, uint32_t count) {
  auto g = GgufFile::Open(path);
  if (g == nullptr || count == 0) return nullptr;
  std::unique_ptr<OlmoeModel> m(new OlmoeModel());
  m->cfg_ = ParseOlmoeConfig(*g);
  if (first + count > m->cfg_.n_expert) return nullptr;
  m->expert_first_ = first;
  m->expert_count_ = count;
  cudaGetDevice(&m->device_);
  ExpertPick pick;
  pick.first = first;
  pick.count = count;
  if (!UploadTensors(path, *g, pick, &m->tensors_, &m->base_, &m->bytes_)) return nullptr;
  m->ws_.reset(new Workspace(m->cfg_));
  m->ws_->view_ok = BuildView(*m, true, &m->ws_->view);
  return m;
}

OlmoeModel::~OlmoeModel() {
  ws_.reset();
  if (base_ != nullptr) cudaFree(base_);
}

const DTensor* OlmoeModel::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const DTensor* OlmoeModel::layer_tensor(int layer, const std::string& suffix) const {
  return tensor("blk." + std::to_string(layer) + "." + suffix);
}

// ------------------------------------------------------------------ KvCache
KvCache::KvCache(const OlmoeConfig& cfg, int max_seq) : max_seq_(max_seq) {
  const size_t dkv = static_cast<size_t>(cfg.n_head_kv) * cfg.head_dim();
  const size_t per = dkv * static_cast<size_t>(max_seq);
  const size_t L = cfg.n_layers;
  if (cudaMalloc(&base_, std::max<size_t>(1, 2 * L * per) * sizeof(float)) != cudaSuccess) {
    base_ = nullptr;
    return;
  }
  cudaMemset(base_, 0, 2 * L * per * sizeof(float));
  float* p = static_cast<float*>(base_);
  for (size_t l = 0; l < L; ++l) {
    k_.push_back(p + (2 * l) * per);
    v_.push_back(p + (2 * l + 1) * per);
  }
}

KvCache::~KvCache() {
  if (base_ != nullptr) cudaFree(base_);
}

// ------------------------------------------------------------------ ExpertReader
std::unique_ptr<ExpertReader> ExpertReader::Open(const std::string& gguf_path) {
  auto g = GgufFile::Open(gguf_path);
  if (g == nullptr) return nullptr;
  std::unordered_map<std::string, Info> info;
  for (const GgufTensorInfo& t : g->tensors()) {
    Info in;
    in.file_offset = t.offset;
    in.expert_bytes = t.nb[2];
    in.n_experts = static_cast<int>(t.ne[2]);
    in.type = t.type;
    info[t.name] = in;
  }
  auto src = TensorSource::Open(gguf_path);
  if (src == nullptr) return nullptr;
  return std::unique_ptr<ExpertReader>(new ExpertReader(std::move(src), std::move(info)));
}

size_t ExpertReader::ExpertBytes(const std::string& name) const {
  auto it = info_.find(name);
  return it == info_.end() ? 0 : it->second.expert_bytes;
}
int ExpertReader::NumExperts(const std::string& name) const {
  auto it = info_.find(name);
  return it == info_.end() ? 0 : it->second.n_experts;
}
int32_t ExpertReader::ExpertType(const std::string& name) const {
  auto it = info_.find(name);
  return it == info_.end() ? -1 : it->second.type;
}
bool ExpertReader::ReadExpert(const std::string& name, int expert_idx, void* out) const {
  auto it = info_.find(name);
  if (it == info_.end()) return false;
  const Info& in = it->second;
  if (expert_idx < 0 || expert_idx >= in.n_experts) return false;
  if (fail_after_ == 0) return false;
  if (fail_after_ > 0) --fail_after_;
  return src_->ReadAt(in.file_offset + static_cast<size_t>(expert_idx) * in.expert_bytes, in.expert_bytes, out);
}

// ------------------------------------------------------------------ StreamingModel
std::unique_ptr<StreamingModel> StreamingModel::Load(const std::string& path, bool pinned_store) {
  auto g = GgufFile::Open(path);
  if (g == nullptr) return nullptr;
  std::unique_ptr<StreamingModel> m(new StreamingModel());
  m->cfg_ = ParseOlmoeConfig(*g);
  ExpertPick none;
  none.skip = true;
  if (!UploadTensors(path, *g, none, &m->tensors_, &m->base_, &m->bytes_)) return nullptr;
  m->reader_ = ExpertReader::Open(path);
  if (m->reader_ == nullptr) return nullptr;
  const OlmoeConfig& c = m->cfg_;
  m->stores_.assign(c.n_layers, ExpertHostStore());
  if (pinned_store) {
    size_t total = 0;
    for (const GgufTensorInfo& t : g->tensors())
      if (IsExpertTensor(t.name)) total += AlignUp(t.nbytes, 64);
    if (total > 0) {
      if (cudaHostAlloc(&m->host_, total, cudaHostAllocDefault) != cudaSuccess) return nullptr;
      auto src = TensorSource::Open(path);
      if (src == nullptr) return nullptr;
      size_t off = 0;
      std::unordered_map<std::string, const uint8_t*> where;
      for (const GgufTensorInfo& t : g->tensors()) {
        if (!IsExpertTensor(t.name)) continue;
        uint8_t* dst = static_cast<uint8_t*>(m->host_) + off;
        if (!src->ReadAt(t.offset, t.nbytes, dst)) return nullptr;
        where[t.name] = dst;
        off += AlignUp(t.nbytes, 64);
      }
      for (uint32_t l = 0; l < c.n_layers; ++l) {
        const std::string b = "blk." + std::to_string(l) + ".";
        ExpertHostStore& s = m->stores_[l];
        const GgufTensorInfo *gt = g->tensor(b + "ffn_gate_exps.weight"), *ut = g->tensor(b + "ffn_up_exps.weight"),
                             *dt = g->tensor(b + "ffn_down_exps.weight");
        if (gt == nullptr || ut == nullptr || dt == nullptr) continue;
        s.gate = where[gt->name];
        s.up = where[ut->name];
        s.down = where[dt->name];
        s.gate_bytes = gt->nb[2];
        s.up_bytes = ut->nb[2];
        s.down_bytes = dt->nb[2];
        s.gate_type = gt->type;
        s.up_type = ut->type;
        s.down_type = dt->type;
        s.n_experts = static_cast<int>(gt->ne[2]);
      }
    }
  }
  m->ws_.reset(new Workspace(c));
  m->ws_->view_ok = BuildView(*m, false, &m->ws_->view);
  cudaStreamCreateWithFlags(&m->ws_->copy_stream, cudaStreamNonBlocking);
  return m;
}

StreamingModel::~StreamingModel() {
  // The slot pools synchronise on the copy stream when released: free them first.
  if (ws_ != nullptr) ws_->slots.caches.clear();
  if (ws_ != nullptr && ws_->copy_stream != nullptr) cudaStreamDestroy(ws_->copy_stream);
  ws_.reset();
  if (base_ != nullptr) cudaFree(base_);
  if (host_ != nullptr) cudaFreeHost(host_);
}

const DTensor* StreamingModel::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const DTensor* StreamingModel::layer_tensor(int layer, const std::string& suffix) const {
  return tensor("blk." + std::to_string(layer) + "." + suffix);
}

const ExpertHostStore* StreamingModel::host_store(int layer) const {
  if (layer < 0 || layer >= static_cast<int>(stores_.size()) || stores_[layer].gate == nullptr) return nullptr;
  return &stores_[layer];
}

}  // namespace nuthatch
