// Routing trace records and file formats (reference: src/trace/routing_trace.h:11-34;
// implemented in csrc/host/trace_io.cc).
// Binary format: magic "NUTHTRC1", u32 version 1, u32 n_layers, u32 n_expert,
// u64 record count, then per record u32 token, u32 layer, u32 n, n x u32
// expert ids; native byte order (routing_trace.cc:14-43).  Text format: one
// record per line, "<layer> e0 e1 ...", token = line order, n_layers and
// n_expert inferred as max+1 (routing_trace.cc:84-111).
#ifndef NUTHATCH_B200_ROUTING_TRACE_H_
#define NUTHATCH_B200_ROUTING_TRACE_H_

#include <cstdint>
#include <string>
#include <vector>

namespace nuthatch {

struct RoutingRecord {
  uint32_t token;
  uint32_t layer;
  std::vector<uint32_t> experts;
};

struct RoutingTrace {
  uint32_t n_layers = 0;
  uint32_t n_expert = 0;
  std::vector<RoutingRecord> records;
};

bool WriteRoutingTrace(const RoutingTrace& trace, const std::string& path);
// False on a missing file, bad magic or version, truncation, or a record whose
// expert count exceeds n_expert (when n_expert > 0).
bool ReadRoutingTrace(const std::string& path, RoutingTrace* out);
// False when no record could be read.
bool ReadRoutingTraceText(const std::string& path, RoutingTrace* out);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_ROUTING_TRACE_H_
