// Routing-trace files: the binary and text formats of the reference's
// src/trace/routing_trace.cc:28-111 (layout in routing_trace.h).  Files are
// read whole into memory and decoded by one pass of a bounds-checked cursor;
// the writer encodes into one buffer and writes it with a single call.
#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstring>
#include <limits>

#include "nuthatch/routing_trace.h"

namespace nuthatch {

namespace {

constexpr char kTraceMagic[8] = {'N', 'U', 'T', 'H', 'T', 'R', 'C', '1'};
constexpr uint32_t kTraceVersion = 1;
// Smallest encoding of one record: token, layer and an expert count of 0.
constexpr uint64_t kMinRecordBytes = 12;

bool Slurp(const std::string& path, std::vector<uint8_t>* bytes) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  bytes->clear();
  uint8_t chunk[1 << 16];
  size_t got = 0;
  while ((got = std::fread(chunk, 1, sizeof(chunk), f)) > 0) bytes->insert(bytes->end(), chunk, chunk + got);
  const bool ok = std::ferror(f) == 0;
  std::fclose(f);
  return ok;
}

// Little cursor over a byte range; every Take fails once the range is short.
struct Cursor {
  const uint8_t* at;
  const uint8_t* end;
  uint64_t left() const { return static_cast<uint64_t>(end - at); }
  template <typename T>
  bool Take(T* v) {
    if (left() < sizeof(T)) return false;
    std::memcpy(v, at, sizeof(T));
    at += sizeof(T);
    return true;
  }
};

template <typename T>
void Append(std::vector<uint8_t>* buf, T v) {
  const size_t at = buf->size();
  buf->resize(at + sizeof(T));
  std::memcpy(buf->data() + at, &v, sizeof(T));
}

// One unsigned decimal field of a text line, as stream extraction into a
// uint32_t reads it: leading blanks skipped, an optional '+', digits; no
// digits or a value beyond 32 bits ends the line.
bool NextField(const char*& p, const char* end, uint32_t* out) {
  while (p < end && std::isspace(static_cast<unsigned char>(*p))) ++p;
  if (p < end && *p == '+') ++p;
  if (p >= end || !std::isdigit(static_cast<unsigned char>(*p))) return false;
  uint64_t v = 0;
  while (p < end && std::isdigit(static_cast<unsigned char>(*p))) {
    v = v * 10 + static_cast<uint64_t>(*p - '0');
    if (v > std::numeric_limits<uint32_t>::max()) return false;
    ++p;
  }
  *out = static_cast<uint32_t>(v);
  return true;
}

}  // namespace

bool WriteRoutingTrace(const RoutingTrace& trace, const std::string& path) {
  std::vector<uint8_t> buf(kTraceMagic, kTraceMagic + sizeof(kTraceMagic));
  Append<uint32_t>(&buf, kTraceVersion);
  Append<uint32_t>(&buf, trace.n_layers);
  Append<uint32_t>(&buf, trace.n_expert);
  Append<uint64_t>(&buf, trace.records.size());
  for (const RoutingRecord& r : trace.records) {
    Append<uint32_t>(&buf, r.token);
    Append<uint32_t>(&buf, r.layer);
    Append<uint32_t>(&buf, static_cast<uint32_t>(r.experts.size()));
    const size_t at = buf.size();
    buf.resize(at + 4 * r.experts.size());
    if (!r.experts.empty()) std::memcpy(buf.data() + at, r.experts.data(), 4 * r.experts.size());
  }
  FILE* f = std::fopen(path.c_str(), "wb");
  if (f == nullptr) return false;
  const bool wrote = std::fwrite(buf.data(), 1, buf.size(), f) == buf.size();
  return (std::fclose(f) == 0) && wrote;
}

bool ReadRoutingTrace(const std::string& path, RoutingTrace* out) {
  std::vector<uint8_t> bytes;
  if (!Slurp(path, &bytes)) return false;
  Cursor c{bytes.data(), bytes.data() + bytes.size()};
  char magic[sizeof(kTraceMagic)];
  if (c.left() < sizeof(magic)) return false;
  std::memcpy(magic, c.at, sizeof(magic));
  c.at += sizeof(magic);
  uint32_t version = 0;
  RoutingTrace t;
  uint64_t n_records = 0;
  if (std::memcmp(magic, kTraceMagic, sizeof(magic)) != 0 || !c.Take(&version) || version != kTraceVersion ||
      !c.Take(&t.n_layers) || !c.Take(&t.n_expert) || !c.Take(&n_records))
    return false;
  // A count the remaining bytes cannot hold is a truncated file.
  if (n_records > c.left() / kMinRecordBytes) return false;
  t.records.resize(n_records);
  for (RoutingRecord& r : t.records) {
    uint32_t n = 0;
    if (!c.Take(&r.token) || !c.Take(&r.layer) || !c.Take(&n)) return false;
    if ((t.n_expert != 0 && n > t.n_expert) || c.left() / 4 < n) return false;
    r.experts.resize(n);
    if (n != 0) std::memcpy(r.experts.data(), c.at, 4ull * n);
    c.at += 4ull * n;
  }
  *out = std::move(t);
  return true;
}

bool ReadRoutingTraceText(const std::string& path, RoutingTrace* out) {
  std::vector<uint8_t> bytes;
  if (!Slurp(path, &bytes)) return false;
  RoutingTrace t;
  uint32_t next_token = 0, max_layer = 0, max_expert = 0;
  const char* p = reinterpret_cast<const char*>(bytes.data());
  const char* const file_end = p + bytes.size();
  while (p < file_end) {
    const char* eol = static_cast<const char*>(std::memchr(p, '\n', static_cast<size_t>(file_end - p)));
    const char* line_end = eol != nullptr ? eol : file_end;
    RoutingRecord r;
    // A line whose first field is a layer number consumes a token number
    // even when no expert follows (such a line is then dropped).
    if (NextField(p, line_end, &r.layer)) {
      r.token = next_token++;
      uint32_t e = 0;
      while (NextField(p, line_end, &e)) r.experts.push_back(e);
      if (!r.experts.empty()) {
        max_layer = std::max(max_layer, r.layer);
        for (uint32_t x : r.experts) max_expert = std::max(max_expert, x);
        t.records.push_back(std::move(r));
      }
    }
    p = eol != nullptr ? eol + 1 : file_end;
  }
  if (t.records.empty()) return false;
  t.n_layers = max_layer + 1;
  t.n_expert = max_expert + 1;
  *out = std::move(t);
  return true;
}

}  // namespace nuthatch
