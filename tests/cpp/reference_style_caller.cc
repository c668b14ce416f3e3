// A caller written against the reference's C++ API (src/tokenizer/tokenizer.h,
// src/model/olmoe_model.h, src/trace/routing_trace.h, src/cache/*.h): the
// same names and calls a nuthatch program makes, compiled here against
// include/nuthatch/ and linked with libnuthatch_b200.so.  Host-only calls
// (no GPU needed).  tests/test_dropin_cpp_cpu.py builds and runs it and
// compares its lines with the Python mirror.
//
//   reference_style_caller <tokenizer.gguf> <trace.bin> <text...>
#include <cstdio>
#include <string>
#include <vector>

#include "nuthatch/cache_policy.h"
#include "nuthatch/olmoe_model.h"
#include "nuthatch/routing_trace.h"
#include "nuthatch/tokenizer.h"

int main(int argc, char** argv) {
  if (argc < 4) {
    std::fprintf(stderr, "usage: %s tokenizer.gguf trace.bin text...\n", argv[0]);
    return 1;
  }
  auto tok = nuthatch::Tokenizer::Load(argv[1]);
  if (tok == nullptr) return 2;
  std::string text;
  for (int i = 3; i < argc; ++i) {
    if (i > 3) text += ' ';
    text += argv[i];
  }
  const std::vector<int32_t> ids = tok->Encode(text);
  std::printf("vocab %lld\nids", static_cast<long long>(tok->vocab_size()));
  for (int32_t t : ids) std::printf(" %d", t);
  std::printf("\ntext %s\n", tok->Decode(ids).c_str());

  // A missing model file gives nullptr, as the reference's factory does.
  std::printf("model %s\n", nuthatch::OlmoeModel::Load("/no/such/model.gguf") == nullptr ? "null" : "loaded");

  // A routing trace of 3 layers x 12 tokens, written and read back.
  nuthatch::RoutingTrace tr;
  tr.n_layers = 3;
  tr.n_expert = 8;
  for (uint32_t t = 0; t < 12; ++t)
    for (uint32_t l = 0; l < 3; ++l) tr.records.push_back({t, l, {(t + l) % 8, (3 * t + 1) % 8, (t * t) % 8}});
  if (!nuthatch::WriteRoutingTrace(tr, argv[2])) return 3;
  nuthatch::RoutingTrace back;
  if (!nuthatch::ReadRoutingTrace(argv[2], &back) || back.records.size() != tr.records.size()) return 4;

  nuthatch::LruPolicy lru(back.n_layers, 3);
  nuthatch::OsPageCachePolicy os(9);
  nuthatch::LearnedPinPolicy learned(back.n_layers, 2, 1, nuthatch::BuildUsage(back));
  const nuthatch::ReplayStats a = nuthatch::Replay(back, &lru);
  const nuthatch::ReplayStats b = nuthatch::Replay(back, &os);
  const nuthatch::ReplayStats c = nuthatch::Replay(back, &learned);
  std::printf("replay %llu %llu %llu of %llu\n", static_cast<unsigned long long>(a.hits),
              static_cast<unsigned long long>(b.hits), static_cast<unsigned long long>(c.hits),
              static_cast<unsigned long long>(a.accesses));
  for (const nuthatch::SweepRow& r : nuthatch::SweepBudgets(back, {2, 4}))
    std::printf("sweep %u %.6f %.6f %.6f\n", r.budget, r.learned, r.lru, r.os);
  return 0;
}
