// Internal: the per-model device workspaces.
#pragma once

#include "engine.h"
#include "nuthatch/olmoe_model.h"
#include "nuthatch/streaming_model.h"

namespace nuthatch {

struct OlmoeModel::Workspace {
  explicit Workspace(const OlmoeConfig& cfg) : engine(cfg) {}
  Engine engine;
  ModelView view;
  bool view_ok = false;
};

struct StreamingModel::Workspace {
  explicit Workspace(const OlmoeConfig& cfg) : engine(cfg) {}
  Engine engine;
  ModelView view;
  bool view_ok = false;
  cudaStream_t copy_stream = nullptr;
  SlotSet slots;  // slot pools kept between StreamingGenerate calls
};

}  // namespace nuthatch
