// C shim over the reference's qwen3/model.cpp, compiled together with that
// file (from the reference tree, in place) into oracle/_ref/libref_model.so.
// Test infrastructure only: it lets the CPU tests pin this repository's
// codecs and loader behaviour against the reference's own implementation.
#include "model.hpp"

#include <cstring>
#include <exception>
#include <string>

namespace {
thread_local std::string g_error;
}

extern "C" {

uint16_t ref_float_to_bf16(float value) { return qwen3::float_to_bf16(value); }
float ref_bf16_to_float(uint16_t value) { return qwen3::bf16_to_float(value); }

// 0 when the reference accepts model_dir/config.json, 1 otherwise.
int ref_validate_config(const char *model_dir) {
  try {
    (void)qwen3::load_and_validate_config(model_dir);
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

// 0 when the reference accepts the whole checkpoint; *arena_size receives
// the 4 KiB-aligned arena size it computes.
int ref_validate_checkpoint(const char *model_dir, uint64_t *arena_size) {
  try {
    const qwen3::Checkpoint c = qwen3::load_and_validate_checkpoint(model_dir);
    if (arena_size) *arena_size = c.arena_size;
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

uint32_t ref_expected_tensor_count(void) {
  return static_cast<uint32_t>(qwen3::expected_tensor_names().size());
}

const char *ref_last_error(void) { return g_error.c_str(); }
}
