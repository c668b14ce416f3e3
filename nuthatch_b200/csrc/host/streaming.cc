// HBM expert slot pool (reference: src/model/expert_slot_cache.cc) and the
// two-phase streaming driver (reference: src/model/streaming_forward.cc).
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <unordered_set>

#include "nuthatch/expert_reader.h"
#include "nuthatch/expert_slot_cache.h"
#include "nuthatch/gguf_file.h"
#include "nuthatch/streaming_forward.h"
#include "workspace.h"

namespace nuthatch {

namespace {
size_t AlignUp(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

std::unique_ptr<ExpertSlotCache> ExpertSlotCache::Create(const OlmoeConfig& cfg, int layer, int capacity,
                                                         ExpertReader* reader, const ExpertHostStore* store,
                                                         const SlotCacheOptions& opt) {
  if (capacity <= 0 || (reader == nullptr && store == nullptr)) return nullptr;
  std::unique_ptr<ExpertSlotCache> c(new ExpertSlotCache());
  const std::string pfx = "blk." + std::to_string(layer) + ".";
  c->gate_name_ = pfx + "ffn_gate_exps.weight";
  c->up_name_ = pfx + "ffn_up_exps.weight";
  c->down_name_ = pfx + "ffn_down_exps.weight";
  int32_t gt, ut, dt;
  size_t gb, ub, db;
  int n_experts;
  if (store != nullptr) {
    c->store_ = *store;
    c->has_store_ = true;
    gt = store->gate_type;
    ut = store->up_type;
    dt = store->down_type;
    gb = store->gate_bytes;
    ub = store->up_bytes;
    db = store->down_bytes;
    n_experts = store->n_experts;
  } else {
    gt = reader->ExpertType(c->gate_name_);
    ut = reader->ExpertType(c->up_name_);
    dt = reader->ExpertType(c->down_name_);
    gb = reader->ExpertBytes(c->gate_name_);
    ub = reader->ExpertBytes(c->up_name_);
    db = reader->ExpertBytes(c->down_name_);
    n_experts = reader->NumExperts(c->gate_name_);
  }
  if (gt < 0 || ut < 0 || dt < 0 || gb == 0 || ub == 0 || db == 0) return nullptr;
  c->reader_ = reader;
  c->capacity_ = capacity;
  c->policy_ = opt.policy;
  c->staging_ = opt.staging > 0 ? opt.staging : 0;
  c->copy_stream_ = opt.copy_stream;
  if (opt.policy == SlotPolicy::kLearnedPin) {
    c->pin_count_ = static_cast<int>(std::min<uint32_t>(opt.pin_slots, static_cast<uint32_t>(capacity)));
  }
  c->lru_slots_ = capacity - c->pin_count_;
  const int slots = capacity + c->staging_;
  // Slot strides keep every slot 256-byte aligned; 256 bytes of tail padding
  // cover the kernels' rounded 16-byte row staging.
  const size_t gs = AlignUp(gb, 256), us = AlignUp(ub, 256), ds = AlignUp(db, 256);
  const size_t total = (gs + us + ds) * slots + 256;
  if (cudaMalloc(&c->base_, total) != cudaSuccess) {
    c->base_ = nullptr;
    return nullptr;
  }
  // Zero the pool on the copy stream so that the preload fills below are
  // ordered after it (the copy stream does not wait for the legacy stream).
  if (cudaMemsetAsync(c->base_, 0, total, static_cast<cudaStream_t>(c->copy_stream_)) != cudaSuccess) return nullptr;
  uint8_t* p = static_cast<uint8_t*>(c->base_);
  auto init = [&](DTensor& t, const std::string& name, int32_t type, size_t stride, int64_t ne0, int64_t ne1,
                  uint8_t* data) {
    t.name = name;
    t.type = type;
    t.ne[0] = ne0;
    t.ne[1] = ne1;
    t.ne[2] = slots;
    t.nb[1] = RowBytes(type, ne0);
    t.nb[2] = stride;
    t.data = data;
    t.nbytes = stride * slots;
  };
  init(c->gate_, c->gate_name_, gt, gs, cfg.n_embd, cfg.n_ff, p);
  init(c->up_, c->up_name_, ut, us, cfg.n_embd, cfg.n_ff, p + gs * slots);
  init(c->down_, c->down_name_, dt, ds, cfg.n_ff, cfg.n_embd, p + (gs + us) * slots);
  c->slot_to_id_.assign(slots, -1);
  c->slot_tick_.assign(slots, 0);
  if (!c->has_store_) {
    for (int i = 0; i < kBounce; ++i) {
      if (cudaHostAlloc(&c->bounce_[i], gb + ub + db, cudaHostAllocDefault) != cudaSuccess ||
          cudaEventCreateWithFlags(reinterpret_cast<cudaEvent_t*>(&c->bounce_done_[i]), cudaEventDisableTiming) !=
              cudaSuccess)
        return nullptr;
    }
  }
  cudaEventCreateWithFlags(reinterpret_cast<cudaEvent_t*>(&c->fill_event_), cudaEventDisableTiming);
  // Learned pin: preload the hottest experts into the pinned slots.
  if (c->pin_count_ > 0 && opt.usage != nullptr) {
    const std::vector<uint32_t> hot = PinnedExperts(*opt.usage, static_cast<uint32_t>(layer),
                                                    static_cast<uint32_t>(c->pin_count_));
    int s = 0;
    for (uint32_t e : hot) {
      if (static_cast<int>(e) >= n_experts) continue;
      if (!c->Fill(s, static_cast<int>(e))) return nullptr;
      c->pinned_[static_cast<int>(e)] = s;
      c->slot_to_id_[s] = static_cast<int>(e);
      ++s;
    }
    cudaStreamSynchronize(static_cast<cudaStream_t>(c->copy_stream_));
  }
  return c;
}

ExpertSlotCache::~ExpertSlotCache() {
  if (copy_stream_ != nullptr) cudaStreamSynchronize(static_cast<cudaStream_t>(copy_stream_));
  else cudaDeviceSynchronize();
  if (fill_event_ != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(fill_event_));
  if (base_ != nullptr) cudaFree(base_);
  for (int i = 0; i < kBounce; ++i) {
    if (bounce_[i] != nullptr) cudaFreeHost(bounce_[i]);
    if (bounce_done_[i] != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(bounce_done_[i]));
  }
}

void ExpertSlotCache::Restart() {
  if (copy_stream_ != nullptr) cudaStreamSynchronize(static_cast<cudaStream_t>(copy_stream_));
  else cudaDeviceSynchronize();
  id_to_slot_.clear();
  for (size_t s = 0; s < slot_to_id_.size(); ++s) {
    if (static_cast<int>(s) >= pin_count_) slot_to_id_[s] = -1;
    slot_tick_[s] = 0;
  }
  tick_ = 0;
  pending_.clear();
  hits_ = misses_ = 0;
  h2d_bytes_ = 0;
  ok_ = true;
}

// Enqueues the three copies of `expert` into `slot` on the copy stream.
bool ExpertSlotCache::Fill(int slot, int expert) {
  cudaStream_t st = static_cast<cudaStream_t>(copy_stream_);
  uint8_t* g = static_cast<uint8_t*>(gate_.data) + gate_.nb[2] * slot;
  uint8_t* u = static_cast<uint8_t*>(up_.data) + up_.nb[2] * slot;
  uint8_t* d = static_cast<uint8_t*>(down_.data) + down_.nb[2] * slot;
  if (has_store_) {
    if (expert < 0 || expert >= store_.n_experts) return false;
    const bool ok =
        cudaMemcpyAsync(g, store_.gate + store_.gate_bytes * expert, store_.gate_bytes, cudaMemcpyHostToDevice, st) ==
            cudaSuccess &&
        cudaMemcpyAsync(u, store_.up + store_.up_bytes * expert, store_.up_bytes, cudaMemcpyHostToDevice, st) ==
            cudaSuccess &&
        cudaMemcpyAsync(d, store_.down + store_.down_bytes * expert, store_.down_bytes, cudaMemcpyHostToDevice, st) ==
            cudaSuccess;
    if (ok) h2d_bytes_ += store_.gate_bytes + store_.up_bytes + store_.down_bytes;
    return ok;
  }
  // Disk -> the next pinned bounce buffer of the ring -> HBM.  The buffer's
  // previous copies must have left it before the disk read overwrites it.
  const int i = bounce_next_;
  bounce_next_ = (bounce_next_ + 1) % kBounce;
  cudaEvent_t done = static_cast<cudaEvent_t>(bounce_done_[i]);
  if (cudaEventSynchronize(done) != cudaSuccess) return false;
  const size_t gb = reader_->ExpertBytes(gate_name_), ub = reader_->ExpertBytes(up_name_),
               db = reader_->ExpertBytes(down_name_);
  uint8_t* b = static_cast<uint8_t*>(bounce_[i]);
  if (!reader_->ReadExpert(gate_name_, expert, b) || !reader_->ReadExpert(up_name_, expert, b + gb) ||
      !reader_->ReadExpert(down_name_, expert, b + gb + ub))
    return false;
  const bool ok = cudaMemcpyAsync(g, b, gb, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                  cudaMemcpyAsync(u, b + gb, ub, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                  cudaMemcpyAsync(d, b + gb + ub, db, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                  cudaEventRecord(done, st) == cudaSuccess;
  if (ok) h2d_bytes_ += gb + ub + db;
  return ok;
}

// LRU part: an empty slot first, else the least recently used one
// (expert_slot_cache.cc:59-72).  Returns -1 when there are no LRU slots.
int ExpertSlotCache::AcquireLru() {
  if (lru_slots_ <= 0) return -1;
  const int b = pin_count_, e = pin_count_ + lru_slots_;
  for (int s = b; s < e; ++s)
    if (slot_to_id_[s] < 0) return s;
  int victim = b;
  for (int s = b + 1; s < e; ++s)
    if (slot_tick_[s] < slot_tick_[victim]) victim = s;
  id_to_slot_.erase(slot_to_id_[victim]);
  slot_to_id_[victim] = -1;
  return victim;
}

std::unordered_map<int, int> ExpertSlotCache::Ensure(const std::vector<int>& expert_ids) {
  std::unordered_map<int, int> result;
  pending_.clear();
  ok_ = true;
  // Distinct non-pinned ids of this batch: when they fit in the LRU part no
  // access can evict an expert this batch still needs, and misses load
  // straight into their slot; otherwise they go through staging slots.
  std::vector<int> distinct;
  {
    std::unordered_set<int> seen;
    for (int id : expert_ids)
      if (seen.insert(id).second && !pinned_.count(id)) distinct.push_back(id);
  }
  const bool direct = static_cast<int>(distinct.size()) <= lru_slots_;
  int next_stage = capacity_;
  for (int id : expert_ids) {
    if (result.count(id)) continue;
    auto pin = pinned_.find(id);
    if (pin != pinned_.end()) {
      ++hits_;
      result[id] = pin->second;
      continue;
    }
    auto it = id_to_slot_.find(id);
    if (it != id_to_slot_.end()) {
      ++hits_;
      slot_tick_[it->second] = ++tick_;
      result[id] = it->second;
      continue;
    }
    ++misses_;
    const int lru = AcquireLru();
    if (direct && lru >= 0) {
      if (!Fill(lru, id)) {
        // A failed fill leaves the slot empty (AcquireLru already unmapped
        // its previous expert), so no later request takes its bytes for id.
        ok_ = false;
        result[id] = lru;
        continue;
      }
      slot_to_id_[lru] = id;
      id_to_slot_[id] = lru;
      slot_tick_[lru] = ++tick_;
      result[id] = lru;
      continue;
    }
    // Staged: the compute reads the staging slot; the expert joins the LRU
    // part (if it has slots) by a device copy after the compute.
    if (next_stage >= capacity_ + staging_) {
      ok_ = false;  // more misses in one batch than staging slots
      result[id] = capacity_;
      continue;
    }
    const int st = next_stage++;
    result[id] = st;
    if (!Fill(st, id)) {
      ok_ = false;  // the expert does not join the LRU part either
      continue;
    }
    if (lru >= 0) {
      slot_to_id_[lru] = id;
      id_to_slot_[id] = lru;
      slot_tick_[lru] = ++tick_;
      pending_.push_back({st, lru});
    }
  }
  cudaEventRecord(static_cast<cudaEvent_t>(fill_event_), static_cast<cudaStream_t>(copy_stream_));
  return result;
}

int ExpertSlotCache::Commit(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Only the last writer of each LRU slot matters.
  std::unordered_map<int, int> last;
  for (auto& pr : pending_) last[pr.second] = pr.first;
  for (auto& pr : pending_) {
    if (last[pr.second] != pr.first) continue;
    const int st = pr.first, dst = pr.second;
    if (slot_to_id_[dst] < 0) continue;
    const DTensor* ts[3] = {&gate_, &up_, &down_};
    for (const DTensor* t : ts) {
      uint8_t* b = static_cast<uint8_t*>(t->data);
      if (cudaMemcpyAsync(b + t->nb[2] * dst, b + t->nb[2] * st, t->nb[2], cudaMemcpyDeviceToDevice, s) !=
          cudaSuccess)
        return NH_E_CUDA;
    }
  }
  pending_.clear();
  return NH_OK;
}

// Longest host wait for one layer's selection before the step is abandoned
// (a healthy phase A takes tens of microseconds).
constexpr double kSelectionTimeoutS = 30.0;

// ------------------------------------------------------------------ driver
std::vector<int32_t> StreamingGenerateEx(const StreamingModel& model, const std::vector<int32_t>& ids, int n_predict,
                                         bool norm_topk, int capacity, const StreamingOptions& opt) {
  std::vector<int32_t> out;
  StreamingStats local;
  StreamingStats& stats = opt.stats != nullptr ? *opt.stats : local;
  stats.status = NH_OK;
  if (ids.empty() || n_predict <= 0) return out;
  StreamingModel::Workspace* ws = model.workspace();
  const OlmoeConfig& c = model.config();
  if (ws == nullptr || !ws->view_ok || capacity <= 0) {
    stats.status = capacity <= 0 ? NH_E_ARG : NH_E_STATE;
    return out;
  }
  for (int32_t t : ids) {
    if (t < 0 || static_cast<uint32_t>(t) >= c.n_vocab) {
      stats.status = NH_E_ARG;
      return out;
    }
  }
  const int L = static_cast<int>(c.n_layers), K = static_cast<int>(c.n_expert_used);
  // The slot pools of the previous call are reused when capacity, policy and
  // pinned set are unchanged: the LRU part restarts empty, the pinned experts
  // stay loaded.  Otherwise they are released and created anew.
  const uint32_t pin_slots = opt.pin_slots > 0 ? opt.pin_slots : LearnedPinSlots(static_cast<uint32_t>(capacity));
  std::vector<std::vector<uint32_t>> pinned;
  if (opt.policy == SlotPolicy::kLearnedPin && opt.usage != nullptr) {
    for (int l = 0; l < L; ++l)
      pinned.push_back(PinnedExperts(*opt.usage, static_cast<uint32_t>(l), std::min<uint32_t>(pin_slots, capacity)));
  }
  StreamingModel::SlotSet& set = ws->slots;
  const bool reuse = set.caches.size() == static_cast<size_t>(L) && set.capacity == capacity &&
                     set.policy == opt.policy && set.pin_slots == pin_slots && set.pinned == pinned;
  if (reuse) {
    for (auto& cache : set.caches) cache->Restart();
  } else {
    set.caches.clear();
    set.capacity = capacity;
    set.policy = opt.policy;
    set.pin_slots = pin_slots;
    set.pinned = pinned;
    for (int l = 0; l < L; ++l) {
      SlotCacheOptions so;
      so.policy = opt.policy;
      so.usage = opt.usage;
      so.pin_slots = pin_slots;
      so.staging = K;
      so.copy_stream = ws->copy_stream;
      set.caches.push_back(ExpertSlotCache::Create(c, l, capacity, model.reader(), model.host_store(l), so));
      if (set.caches.back() == nullptr) {
        set.caches.clear();
        stats.status = NH_E_NOMEM;
        return out;
      }
    }
  }
  std::vector<std::unique_ptr<ExpertSlotCache>>& caches = set.caches;
  Engine& e = ws->engine;
  const int P = static_cast<int>(ids.size());
  int rc = e.Reserve(P + n_predict + 1, P, n_predict, false);
  if (rc == NH_OK) rc = e.Begin(ids.data(), P, n_predict);
  if (opt.trace != nullptr) {
    opt.trace->n_layers = c.n_layers;
    opt.trace->n_expert = c.n_expert;
    opt.trace->records.clear();
  }
  const int steps = P + n_predict - 1;
  cudaStream_t s = e.stream();
  double fill_ms = 0;
  for (int t = 0; t < steps && rc == NH_OK; ++t) {
    rc = e.EnqueueEmbed(ws->view);
    for (int l = 0; l < L && rc == NH_OK; ++l) {
      // Phase A: attention + residual + router; the selected ids come back
      // through mapped host memory (no stream synchronisation).
      rc = e.EnqueueAttnPhase(ws->view, l, norm_topk, false);
      if (rc == NH_OK) rc = e.AwaitSelection(kSelectionTimeoutS);
      if (rc != NH_OK) break;
      const auto t0 = std::chrono::steady_clock::now();
      std::vector<int> sel(e.sel_host(), e.sel_host() + K);
      if (opt.trace != nullptr) {
        RoutingRecord r;
        r.token = static_cast<uint32_t>(t);
        r.layer = static_cast<uint32_t>(l);
        for (int id : sel) r.experts.push_back(static_cast<uint32_t>(id));
        opt.trace->records.push_back(std::move(r));
      }
      // Host slot decisions; misses fill on the copy stream.
      std::unordered_map<int, int> slot = caches[l]->Ensure(sel);
      if (!caches[l]->ok()) {
        rc = NH_E_IO;
        break;
      }
      // The slots travel with the phase B launches (no copy before them).
      for (int i = 0; i < K; ++i) e.wsel_host()[i] = slot[sel[i]];
      if (cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(caches[l]->fills_done_event()), 0) != cudaSuccess) {
        rc = NH_E_CUDA;
        break;
      }
      fill_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
      // Phase B on the slot tensors.
      const ExpertSlotCache& sc = *caches[l];
      rc = e.EnqueueMoePhase(ws->view, l, sc.gate_slots()->data, sc.gate_slots()->type, sc.gate_slots()->nb[2],
                             sc.up_slots()->data, sc.up_slots()->type, sc.up_slots()->nb[2],
                             sc.down_slots()->data, sc.down_slots()->type, sc.down_slots()->nb[2], e.wsel_dev(),
                             false, e.wsel_host());
      if (rc == NH_OK) rc = caches[l]->Commit(s);
    }
    if (rc == NH_OK) rc = e.EnqueueFinal(ws->view, false);
  }
  if (rc == NH_OK) rc = e.Finish(n_predict, &out);
  stats.hits.assign(L, 0);
  stats.misses.assign(L, 0);
  stats.h2d_bytes = 0;
  for (int l = 0; l < L; ++l) {
    stats.hits[l] = caches[l]->hits();
    stats.misses[l] = caches[l]->misses();
    stats.h2d_bytes += caches[l]->h2d_bytes();
  }
  stats.fill_ms = fill_ms;
  if (rc != NH_OK) {
    stats.status = rc;
    cudaStreamSynchronize(s);
    out.clear();
  }
  cudaStreamSynchronize(ws->copy_stream);
  return out;
}

std::vector<int32_t> StreamingGenerate(const StreamingModel& model, std::vector<int32_t> ids, int n_predict,
                                       bool norm_topk, int capacity) {
  return StreamingGenerateEx(model, ids, n_predict, norm_topk, capacity, StreamingOptions());
}

}  // namespace nuthatch
