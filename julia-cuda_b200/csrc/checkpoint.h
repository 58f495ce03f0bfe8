// Checkpoint directories in the reference's layout (src/checkpoint.rs:27-62): model.safetensors
// (the weights), encoder/config.json (the ModernBERT encoder's Hugging Face config) and
// julia_config.json (the head and scorer), read into the raw f32 format the engine prepares
// (julia_cuda.h documents its order). Host code only.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/julia_cuda.h"

namespace jc {

// Reads dir/model.safetensors + dir/encoder/config.json + dir/julia_config.json (+ the optional
// dir/jc_names.json name overrides) into cfg and raw. false with the reason on any inconsistency
// (a missing tensor, a shape that disagrees with the config, an unsupported dtype, a short file).
bool read_checkpoint(const std::string &dir, jc_model_config *cfg, std::vector<float> *raw,
                     std::string *why);

// Writes cfg + raw as such a directory (tensors in dtype 0 F32, 1 F16, 2 BF16 under the default
// names; creates dir/encoder).
bool write_checkpoint(const std::string &dir, const jc_model_config &cfg, const float *raw,
                      int dtype, std::string *why);

// Whether dir holds a safetensors checkpoint.
bool has_checkpoint(const std::string &dir);

}  // namespace jc
