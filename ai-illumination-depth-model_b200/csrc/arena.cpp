// Liveness-based activation arena (src/engine/arena.ts:57-172).
//
// The greedy policy is the reference's: each op's output takes the smallest
// free buffer that fits, else the largest free buffer grows, else a new
// buffer is added; inputs are released after the output is placed, so an op
// never aliases its own source and destination. Keeping the same policy keeps
// the same 7-buffer, 19.03 MB/frame plan, which debugTensor's liveAtEnd
// semantics depend on. Sizes are per frame; the device arena multiplies them
// by the batch.
#include <algorithm>
#include <limits>
#include <sstream>

#include "host.h"

namespace illumina {

namespace {
long tensor_elements(const TensorShape &s) { return (long)s.h * s.w * (s.c / 4); }
bool excluded(const std::vector<std::string> &ex, const std::string &n) {
  return std::find(ex.begin(), ex.end(), n) != ex.end();
}
}  // namespace

ArenaPlan plan_arena(const Architecture &a, const std::vector<std::string> &exclude, bool no_alias) {
  ArenaPlan p;
  std::map<std::string, int> last_read;
  for (size_t i = 0; i < a.ops.size(); i++)
    for (const auto &t : op_inputs(a.ops[i])) last_read[t] = (int)i;
  std::vector<bool> free_;
  std::map<int, std::string> occupant;
  for (size_t i = 0; i < a.ops.size(); i++) {
    const Op &op = a.ops[i];
    if (!excluded(exclude, op.out) && !p.assignment.count(op.out)) {
      long need = tensor_elements(a.shape(op.out));
      int chosen = -1;
      if (!no_alias) {
        long chosen_size = std::numeric_limits<long>::max();
        for (size_t b = 0; b < p.buffer_sizes.size(); b++)
          if (free_[b] && p.buffer_sizes[b] >= need && p.buffer_sizes[b] < chosen_size)
            chosen = (int)b, chosen_size = p.buffer_sizes[b];
        if (chosen == -1) {
          int grow = -1;
          long grow_size = -1;
          for (size_t b = 0; b < p.buffer_sizes.size(); b++)
            if (free_[b] && p.buffer_sizes[b] > grow_size) grow = (int)b, grow_size = p.buffer_sizes[b];
          if (grow != -1) {
            chosen = grow;
            p.buffer_sizes[grow] = need;
          }
        }
      }
      if (chosen == -1) {
        chosen = (int)p.buffer_sizes.size();
        p.buffer_sizes.push_back(need);
        free_.push_back(false);
      }
      free_[chosen] = false;
      p.assignment[op.out] = chosen;
      occupant[chosen] = op.out;
    }
    for (const auto &t : op_inputs(op)) {
      auto lr = last_read.find(t);
      if (lr != last_read.end() && lr->second == (int)i) {
        auto as = p.assignment.find(t);
        if (as != p.assignment.end() && occupant[as->second] == t) free_[as->second] = true;
      }
    }
  }
  for (long n : p.buffer_sizes) p.total_bytes += n * 16;
  for (const auto &n : a.tensor_order)
    if (!excluded(exclude, n)) p.naive_bytes += tensor_elements(a.tensors.at(n)) * 16;
  return p;
}

void validate_arena(const Architecture &a, const ArenaPlan &p, const std::vector<std::string> &exclude) {
  std::map<std::string, int> first_write, last_read;
  for (size_t i = 0; i < a.ops.size(); i++) {
    if (!first_write.count(a.ops[i].out)) first_write[a.ops[i].out] = (int)i;
    for (const auto &t : op_inputs(a.ops[i])) last_read[t] = (int)i;
  }
  std::vector<std::string> names;
  for (const auto &n : a.tensor_order)
    if (!excluded(exclude, n)) names.push_back(n);
  auto get = [](const std::map<std::string, int> &m, const std::string &k, int dflt) {
    auto it = m.find(k);
    return it == m.end() ? dflt : it->second;
  };
  for (const auto &x : names)
    for (const auto &y : names) {
      if (x >= y) continue;
      auto ax = p.assignment.find(x), ay = p.assignment.find(y);
      if (ax == p.assignment.end() || ay == p.assignment.end() || ax->second != ay->second) continue;
      int a0 = get(first_write, x, 0), a1 = get(last_read, x, a0);
      int b0 = get(first_write, y, 0), b1 = get(last_read, y, b0);
      if (a0 <= b1 && b0 <= a1) {
        std::ostringstream m;
        m << "arena: " << x << " [" << a0 << ".." << a1 << "] and " << y << " [" << b0 << ".." << b1
          << "] overlap in buffer " << ax->second;
        throw Error(ILLUMINA_INVALID_ARG, m.str());
      }
    }
  for (const auto &n : names) {
    auto as = p.assignment.find(n);
    if (as == p.assignment.end()) throw Error(ILLUMINA_INVALID_ARG, "arena: " + n + " was never assigned a buffer");
    long need = tensor_elements(a.shape(n));
    if (p.buffer_sizes[as->second] < need)
      throw Error(ILLUMINA_INVALID_ARG, "arena: buffer " + std::to_string(as->second) + " holds " +
                                            std::to_string(p.buffer_sizes[as->second]) + " but " + n + " needs " +
                                            std::to_string(need));
  }
}

std::string arena_to_json(const ArenaPlan &p) {
  std::ostringstream js;
  js << "{\"bufferSizes\":[";
  for (size_t i = 0; i < p.buffer_sizes.size(); i++) js << (i ? "," : "") << p.buffer_sizes[i];
  js << "],\"assignment\":{";
  bool first = true;
  for (const auto &kv : p.assignment) {
    js << (first ? "" : ",") << json_escape(kv.first) << ":" << kv.second;
    first = false;
  }
  js << "},\"totalBytes\":" << p.total_bytes << ",\"naiveBytes\":" << p.naive_bytes << "}";
  return js.str();
}

}  // namespace illumina
