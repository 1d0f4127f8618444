// Definitions of the opaque handles of the C ABI (shared by the translation units that
// implement exports).
#pragma once
#include <vector>

#include "transcribe.h"

struct QwenAsrEngine {
  qasr::Ctx ctx;
};

struct QwenAsrStreamState {
  qasr::StreamState state;
  std::vector<float> audio_buf;  // the reference passes the full accumulated buffer (c_api.rs:171-175)
};
