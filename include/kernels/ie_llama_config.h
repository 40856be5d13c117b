// Llama-3.1-8B shape constants used by the drop-in entry points. Same values
// as the reference's InfEngineConfig (config.h:5-26).
#pragma once

namespace ie_llama {
constexpr int kMaxContextLength = 8192;
constexpr int kVocabSize = 128256;
constexpr int kNumLayers = 32;
constexpr int kHiddenSize = 4096;
constexpr int kNumQHeads = 32;
constexpr int kNumKvHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kFfnDim = 14336;
}  // namespace ie_llama
