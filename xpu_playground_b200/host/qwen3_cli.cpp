// `qwen3` command: greedy generation from a safetensors checkpoint on one
// B200, with the reference program's flags, input format, stopping rule and
// JSON output (qwen3/main.cpp:15-110, 330-370):
//
//   qwen3 --model-dir DIR --input-ids FILE|- --max-new-tokens N [--max-seq-len N]
//         [--device N]
//
// Input ids are whitespace-separated decimal token ids (a file, or stdin for
// "-"); the output is one line {"generated_ids":[...]}; generation stops
// after EOS 151645 or end-of-turn 151643. Errors print "qwen3: <what>" on
// stderr and exit 1. Unlike the reference (Qwen3-8B only, 508 synchronous
// launches per token), any Qwen3 checkpoint with head_dim 128 runs, and
// prompt plus generation run device-resident with one host synchronisation.
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include "xpu_cuda.h"

namespace {

constexpr uint32_t kMaximumContext = 40960;  // qwen3/model.hpp:18

struct Options {
  std::string model_dir, input_ids;
  uint32_t max_new_tokens = 0, max_sequence = kMaximumContext;
  bool has_max_new_tokens = false;
  int device = 0;
};

const char *kUsage = "Usage: qwen3 --model-dir DIR --input-ids FILE|- --max-new-tokens N [--max-seq-len N] [--device N]";

[[noreturn]] void usage_error(const std::string &message) { throw std::runtime_error(message + "\n" + kUsage); }

uint32_t parse_u32(const std::string &text, const std::string &option, bool allow_zero) {
  size_t used = 0;
  unsigned long long v = 0;
  try {
    v = std::stoull(text, &used);
  } catch (...) {
    usage_error("invalid value for " + option + ": " + text);
  }
  if (used != text.size() || text.empty() || text[0] == '-' || v > std::numeric_limits<uint32_t>::max() ||
      (!allow_zero && v == 0))
    usage_error("invalid value for " + option + ": " + text);
  return static_cast<uint32_t>(v);
}

Options parse(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string opt = argv[i];
    if (opt == "-h" || opt == "--help") {
      std::cout << kUsage << '\n';
      std::exit(0);
    }
    if (i + 1 == argc) usage_error("missing value for " + opt);
    const std::string value = argv[++i];
    if (opt == "--model-dir") o.model_dir = value;
    else if (opt == "--input-ids") o.input_ids = value;
    else if (opt == "--max-new-tokens") { o.max_new_tokens = parse_u32(value, opt, true); o.has_max_new_tokens = true; }
    else if (opt == "--max-seq-len") o.max_sequence = parse_u32(value, opt, false);
    else if (opt == "--device") o.device = static_cast<int>(parse_u32(value, opt, true));
    else usage_error("unknown option: " + opt);
  }
  if (o.model_dir.empty()) usage_error("--model-dir is required");
  if (o.input_ids.empty()) usage_error("--input-ids is required");
  if (!o.has_max_new_tokens) usage_error("--max-new-tokens is required");
  if (o.max_sequence > kMaximumContext) usage_error("--max-seq-len cannot exceed 40960");
  return o;
}

std::vector<uint32_t> read_ids(const Options &o, uint32_t vocab) {
  std::ifstream file;
  std::istream *in = &std::cin;
  if (o.input_ids != "-") {
    file.open(o.input_ids);
    if (!file) throw std::runtime_error("cannot open input token file: " + o.input_ids);
    in = &file;
  }
  std::vector<uint32_t> ids;
  std::string tok;
  while (*in >> tok) {
    size_t used = 0;
    unsigned long long v = 0;
    try {
      v = std::stoull(tok, &used);
    } catch (...) {
      throw std::runtime_error("invalid input token ID: " + tok);
    }
    if (used != tok.size() || tok[0] == '-' || v >= vocab)
      throw std::runtime_error("input token ID is outside [0, " + std::to_string(vocab - 1) + "]: " + tok);
    ids.push_back(static_cast<uint32_t>(v));
  }
  if (!in->eof()) throw std::runtime_error("failed while reading input token IDs");
  if (ids.empty()) throw std::runtime_error("at least one input token ID is required");
  if (ids.size() > o.max_sequence || o.max_new_tokens > o.max_sequence - ids.size())
    throw std::runtime_error("prompt plus requested generation exceeds --max-seq-len");
  return ids;
}

void check(int status, const char *what) {
  if (status != XPU_OK) throw std::runtime_error(std::string(what) + ": " + xpu_last_error());
}

}  // namespace

int main(int argc, char **argv) {
  xpu_qwen3_engine *engine = nullptr;
  try {
    const Options o = parse(argc, argv);
    xpu_qwen3_shape shape{};
    check(xpu_qwen3_read_config(o.model_dir.c_str(), &shape), "config");
    const std::vector<uint32_t> prompt = read_ids(o, shape.vocab_size);
    check(xpu_qwen3_create(&shape, o.max_sequence, o.device, 0, 1, &engine), "engine");
    check(xpu_qwen3_load_checkpoint(engine, o.model_dir.c_str()), "checkpoint");
    std::vector<uint32_t> out(o.max_new_tokens ? o.max_new_tokens : 1);
    uint32_t count = 0;
    if (o.max_new_tokens)
      check(xpu_qwen3_generate(engine, prompt.data(), static_cast<uint32_t>(prompt.size()), o.max_new_tokens, 1,
                               out.data(), &count),
            "generate");
    xpu_qwen3_destroy(engine);
    engine = nullptr;
    std::cout << "{\"generated_ids\":[";
    for (uint32_t i = 0; i < count; ++i) std::cout << (i ? "," : "") << out[i];
    std::cout << "]}\n";
    return 0;
  } catch (const std::exception &e) {
    if (engine) xpu_qwen3_destroy(engine);
    std::cerr << "qwen3: " << e.what() << '\n';
    return 1;
  }
}
