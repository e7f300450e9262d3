// lower.h -- the records of a lowering made through the C ABI (tc_lower_json), shared by the emitter
// (lower.cpp) and the runner / resident program (program.cpp).
#pragma once

#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "../../include/tcb200.h"
#include "json.h"

namespace tcl {

using tcb_json::Value;
using i64 = int64_t;

struct Graph;

struct Node {
  int id = 0;
  std::string op;
  std::vector<int> inputs;
  std::vector<i64> shape;
  // attributes
  std::string name;               // input
  int axis = 0;                   // sum, max
  bool keepDims = false;
  std::vector<int> perm;          // transpose
  bool has_value = false;         // const
  bool scalar_value = true;
  double value = 0.0;
  std::vector<double> values;
  std::vector<i64> attr_shape;    // input, const, broadcast, reshape
  std::string kind, pattern;      // fused
  int output = -1;
  std::shared_ptr<Graph> body;
  Value attrs_json;               // the attributes as given (for the one-op cache key)
};

struct Graph {
  std::vector<Node> nodes;
};

// ---------------------------------------------------------------- launch records
struct Map {
  std::string region;
  i64 off, cols, rows, batches, rs, bs, bc, br;
};

struct Call {
  std::string name;
  i64 grid[3], block[3];
  i64 smem = 0;
  std::vector<i64> params;
  std::vector<Map> tma;
  bool has_tma = false;
  i64 err_offset = -1;
  int out_node = -1;
  std::vector<std::pair<int, int>> ptr_params;
};

struct Launch {
  int node = -1;
  std::vector<int> nodes;        // a launch with two outputs lists both
  std::string op, kind, pattern; // pattern empty = none
  bool has_pattern = false;
  std::vector<int> inputs;
  std::string code;
  std::vector<Call> calls;
  i64 scratch_bytes = 0, bytes = 0;
  std::vector<std::pair<std::string, Value>> info;
};

struct Lowering {
  std::shared_ptr<Graph> graph;
  std::vector<Launch> launches;
  std::vector<int> folded;
  std::vector<std::pair<int, int>> transposed;  // (transposeLast2, matmul) computed as one transposed product
  std::map<std::string, Launch> plain_cache;
};


}  // namespace tcl

// The opaque handle of the C ABI.
struct tc_lowered {
  tcl::Lowering L;
  std::string json;   // built on first request
};

