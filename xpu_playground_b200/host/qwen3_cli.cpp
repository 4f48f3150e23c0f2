// `qwen3` command: greedy generation from a safetensors checkpoint on one
// B200. Its flags, input format, stopping rule, messages and JSON output are
// the reference program's interface (qwen3/main.cpp:15-110, 330-370):
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
#include <cctype>
#include <cstdint>
#include <fstream>
#include <iostream>
#include <iterator>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "cli.hpp"
#include "xpu_cuda.h"

namespace {

using namespace xpu_cli;

constexpr uint32_t kMaximumContext = 40960;  // qwen3/model.hpp:18
constexpr const char *kUsage =
    "Usage: qwen3 --model-dir DIR --input-ids FILE|- --max-new-tokens N [--max-seq-len N] [--device N]";

struct Request {
  std::string model_dir, input_ids;
  uint32_t max_new_tokens = 0, max_sequence = kMaximumContext, device = 0;
  bool max_new_tokens_given = false;
};

std::runtime_error usage_error(const std::string &what) { return std::runtime_error(what + "\n" + kUsage); }

// The command line; false after --help.
bool read_request(int argc, char **argv, Request &q) {
  FlagTable t([](std::ostream &out) { out << kUsage << '\n'; });
  uint32_t new_tokens = 0;
  t.lenient_counts()
      .text("--model-dir", &q.model_dir)
      .text("--input-ids", &q.input_ids)
      .count("--max-new-tokens", true, &new_tokens)
      .count("--max-seq-len", false, &q.max_sequence)
      .count("--device", true, &q.device);
  try {
    if (!t.parse(argc, argv)) return false;
  } catch (const FlagError &e) {
    switch (e.problem) {
      case FlagProblem::kNoValue: throw usage_error("missing value for " + e.flag);
      case FlagProblem::kUnknown: throw usage_error("unknown option: " + e.flag);
      default: throw usage_error("invalid value for " + e.flag + ": " + e.value);
    }
  }
  q.max_new_tokens_given = t.given("--max-new-tokens");
  q.max_new_tokens = new_tokens;
  if (q.model_dir.empty()) throw usage_error("--model-dir is required");
  if (q.input_ids.empty()) throw usage_error("--input-ids is required");
  if (!q.max_new_tokens_given) throw usage_error("--max-new-tokens is required");
  if (q.max_sequence > kMaximumContext) throw usage_error("--max-seq-len cannot exceed 40960");
  return true;
}

// One whitespace-free word of the id list -> token id. A word that does not
// start like a number (optional sign, then a digit) or does not fit 64 bits
// is not an id at all; a number with trailing characters, a negative one or
// one past the vocabulary is outside the id range.
uint32_t word_to_id(const std::string &word, uint32_t vocab) {
  const size_t digits_at = (word[0] == '+' || word[0] == '-') ? 1 : 0;
  if (digits_at >= word.size() || !std::isdigit(static_cast<unsigned char>(word[digits_at])))
    throw std::runtime_error("invalid input token ID: " + word);
  size_t end = digits_at;
  while (end < word.size() && std::isdigit(static_cast<unsigned char>(word[end]))) ++end;
  uint64_t value = 0;
  if (!read_count(std::string_view(word).substr(0, end), true, value))
    throw std::runtime_error("invalid input token ID: " + word);
  if (end != word.size() || value >= vocab)
    throw std::runtime_error("input token ID is outside [0, " + std::to_string(vocab - 1) + "]: " + word);
  return static_cast<uint32_t>(value);
}

std::vector<uint32_t> read_prompt(const Request &q, uint32_t vocab) {
  std::string text;
  if (q.input_ids == "-") {
    text.assign(std::istreambuf_iterator<char>(std::cin), std::istreambuf_iterator<char>());
    if (std::cin.bad()) throw std::runtime_error("failed while reading input token IDs");
  } else {
    std::ifstream file(q.input_ids, std::ios::binary);
    if (!file) throw std::runtime_error("cannot open input token file: " + q.input_ids);
    text.assign(std::istreambuf_iterator<char>(file), std::istreambuf_iterator<char>());
    if (file.bad()) throw std::runtime_error("failed while reading input token IDs");
  }
  std::vector<uint32_t> ids;
  size_t at = 0;
  while (true) {
    at = text.find_first_not_of(" \t\n\v\f\r", at);
    if (at == std::string::npos) break;
    const size_t stop = std::min(text.find_first_of(" \t\n\v\f\r", at), text.size());
    ids.push_back(word_to_id(text.substr(at, stop - at), vocab));
    at = stop;
  }
  if (ids.empty()) throw std::runtime_error("at least one input token ID is required");
  if (ids.size() > q.max_sequence || q.max_new_tokens > q.max_sequence - ids.size())
    throw std::runtime_error("prompt plus requested generation exceeds --max-seq-len");
  return ids;
}

void check(int status, const char *what) {
  if (status != XPU_OK) throw std::runtime_error(std::string(what) + ": " + xpu_last_error());
}

// Owns the engine handle for the lifetime of one run.
struct EngineHandle {
  xpu_qwen3_engine *e = nullptr;
  ~EngineHandle() {
    if (e) xpu_qwen3_destroy(e);
  }
};

std::string generate(const Request &q) {
  xpu_qwen3_shape shape{};
  check(xpu_qwen3_read_config(q.model_dir.c_str(), &shape), "config");
  const std::vector<uint32_t> prompt = read_prompt(q, shape.vocab_size);
  EngineHandle engine;
  check(xpu_qwen3_create(&shape, q.max_sequence, static_cast<int>(q.device), 0, 1, &engine.e), "engine");
  check(xpu_qwen3_load_checkpoint(engine.e, q.model_dir.c_str()), "checkpoint");
  std::vector<uint32_t> out(q.max_new_tokens ? q.max_new_tokens : 1);
  uint32_t produced = 0;
  if (q.max_new_tokens)
    check(xpu_qwen3_generate(engine.e, prompt.data(), static_cast<uint32_t>(prompt.size()), q.max_new_tokens, 1,
                             out.data(), &produced),
          "generate");
  std::ostringstream json;
  json << "{\"generated_ids\":[";
  for (uint32_t i = 0; i < produced; ++i) json << (i ? "," : "") << out[i];
  json << "]}\n";
  return json.str();
}

}  // namespace

int main(int argc, char **argv) {
  try {
    Request q;
    if (!read_request(argc, argv, q)) return 0;
    std::cout << generate(q);
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "qwen3: " << e.what() << '\n';
    return 1;
  }
}
