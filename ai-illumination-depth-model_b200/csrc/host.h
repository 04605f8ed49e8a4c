// Host-side runtime of the IlluminaDepth hot path: the layer table, the weight
// container, the seeded initialiser and the arena planner. Pure C++, no CUDA.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "illumina.h"

namespace illumina {

// An error carrying the C-ABI status it maps to.
struct Error : std::runtime_error {
  illumina_status status;
  Error(illumina_status s, const std::string &m) : std::runtime_error(m), status(s) {}
};

void set_last_error(const std::string &msg);

// ---------------------------------------------------------------------------
// Layer table (src/model/arch.ts)
// ---------------------------------------------------------------------------

enum class OpKind { Preprocess, Conv, Pw, Dwpw, Lateral, Head, BilateralUp };

const char *op_kind_name(OpKind k);
const char *act_name(int act);

struct TensorShape {
  int h = 0, w = 0, c = 0;
  long elems() const { return (long)h * w * c; }
};

struct Op {
  OpKind kind;
  std::string name, in, out, residual, coarse, skip;
  int k = 0, stride = 0, act = ILLUMINA_ACT_LINEAR, mid_act = ILLUMINA_ACT_LINEAR;
};

struct Architecture {
  std::string name;
  int input_size = 0;
  double mean[3], std[3];
  std::vector<std::string> tensor_order;  // insertion order, as the JS object
  std::map<std::string, TensorShape> tensors;
  std::vector<Op> ops;
  const TensorShape &shape(const std::string &n) const;
};

// buildArchitecture (arch.ts:191-385). Throws Error(INVALID_ARG) unless
// input_size is a positive multiple of 32.
Architecture build_architecture(int input_size);

struct OpCost {
  std::string name;
  OpKind kind;
  long macs = 0, params = 0;
};
// costOf (arch.ts:415-489)
std::vector<OpCost> cost_of(const Architecture &a, long *total_macs, long *total_params);

// opInputs (src/engine/arena.ts:19-33)
std::vector<std::string> op_inputs(const Op &op);

// ---------------------------------------------------------------------------
// Weights (src/model/weights.ts)
// ---------------------------------------------------------------------------

struct WeightSpec {
  std::string name;
  std::vector<int> shape;
  size_t count = 0;   // elements
  size_t offset = 0;  // element offset in the flat blob
};

// weightSpecs (weights.ts:29-63), with flat-blob offsets.
std::vector<WeightSpec> weight_specs(const Architecture &a);
size_t weight_count(const Architecture &a);

double half_to_float(uint16_t h);
// synthesizeWeights (weights.ts:227-251) into a flat blob.
std::vector<float> synthesize_weights(const Architecture &a, uint32_t seed);
// parseWeights (weights.ts:97-165) into a flat blob. Throws Error.
std::vector<float> parse_weights(const Architecture &a, const uint8_t *bytes, size_t len);
// serializeWeights (weights.ts:168-194).
std::vector<uint8_t> serialize_weights(const Architecture &a, const float *blob, size_t count);

// ---------------------------------------------------------------------------
// Arena (src/engine/arena.ts)
// ---------------------------------------------------------------------------

struct ArenaPlan {
  std::vector<long> buffer_sizes;          // vec4 elements per frame
  std::map<std::string, int> assignment;   // tensor -> buffer
  long total_bytes = 0, naive_bytes = 0;   // fp32, per frame
};

// planArena (arena.ts:57-128). With `no_alias` every tensor gets its own
// buffer (the debug / per-layer parity mode).
ArenaPlan plan_arena(const Architecture &a, const std::vector<std::string> &exclude, bool no_alias = false);
// validateArena (arena.ts:134-172). Throws Error(INVALID_ARG) on a violation.
void validate_arena(const Architecture &a, const ArenaPlan &p, const std::vector<std::string> &exclude);

// JSON renderings for the C ABI.
std::string arch_to_json(const Architecture &a);
std::string arena_to_json(const ArenaPlan &p);

// ---------------------------------------------------------------------------
// Minimal JSON reader (for .idm / .ntb headers)
// ---------------------------------------------------------------------------

struct Json {
  enum Type { Null, Bool, Number, String, Array, Object } type = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // insertion order
  const Json *get(const std::string &k) const;
};

// Parses `text`; throws std::runtime_error with a position on malformed input.
Json parse_json(const std::string &text);
std::string json_escape(const std::string &s);

}  // namespace illumina
