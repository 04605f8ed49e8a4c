// The .idm weight container (src/model/weights.ts:82-194) and the seeded
// Kaiming initialiser (weights.ts:200-251).
//
// The container layout is a format the reference defines and other tools
// write (tools/export/export_idm.py), so it is kept byte for byte: u32 LE
// header length, compact UTF-8 JSON header {"format","arch","tensors":{name:
// {"dtype","shape","offset","length"}}}, then the tight blob in weightSpecs
// order. Validation order and messages follow parseWeights so callers see the
// same errors.
#include <cmath>
#include <cstring>
#include <sstream>

#include "host.h"

namespace illumina {

double half_to_float(uint16_t h) {
  int sign = (h & 0x8000) >> 15;
  int e = (h & 0x7c00) >> 10;
  int frac = h & 0x03ff;
  double v;
  if (e == 0) v = frac * std::ldexp(1.0, -24);
  else if (e == 0x1f) v = frac == 0 ? INFINITY : NAN;
  else v = (frac + 1024) * std::ldexp(1.0, e - 25);
  return sign ? -v : v;
}

namespace {

// mulberry32 (weights.ts:200-209): uint32 state, output in [0, 1).
struct Mulberry32 {
  uint32_t a;
  double next() {
    a += 0x6d2b79f5u;
    uint32_t t = a;
    t = (t ^ (t >> 15)) * (t | 1u);
    t ^= t + (t ^ (t >> 7)) * (t | 61u);
    return (double)(t ^ (t >> 14)) / 4294967296.0;
  }
  // Box-Muller (weights.ts:212-216)
  double gaussian() {
    double u = next();
    if (u < 1e-9) u = 1e-9;
    double v = next();
    return std::sqrt(-2.0 * std::log(u)) * std::cos(2.0 * M_PI * v);
  }
};

bool ends_with(const std::string &s, const std::string &suf) {
  return s.size() >= suf.size() && s.compare(s.size() - suf.size(), suf.size(), suf) == 0;
}

std::string js_number(double v) {
  if (v == std::floor(v) && std::fabs(v) < 1e15) return std::to_string((long long)v);
  std::ostringstream o;
  o.precision(17);
  o << v;
  return o.str();
}

std::string js_string_of(const Json *j) {
  if (!j) return "undefined";
  switch (j->type) {
    case Json::String: return j->str;
    case Json::Number: return js_number(j->num);
    case Json::Bool: return j->b ? "true" : "false";
    case Json::Null: return "null";
    default: return "[object]";
  }
}

}  // namespace

std::vector<float> synthesize_weights(const Architecture &a, uint32_t seed) {
  auto specs = weight_specs(a);
  std::vector<float> blob(weight_count(a), 0.0f);
  Mulberry32 rng{seed};
  for (const auto &s : specs) {
    if (ends_with(s.name, "bias")) continue;  // zeros, no draws
    long fan_in = 1;
    if (s.name.find("dw_weight") != std::string::npos) fan_in = (long)s.shape[1] * s.shape[2];
    else
      for (size_t i = 1; i < s.shape.size(); i++) fan_in *= s.shape[i];
    double stdv = std::sqrt(2.0 / (double)(fan_in > 1 ? fan_in : 1));
    double scale = s.name.rfind("head", 0) == 0 ? stdv * 0.05 : stdv;
    for (size_t j = 0; j < s.count; j++) blob[s.offset + j] = (float)(rng.gaussian() * scale);
  }
  return blob;
}

std::vector<float> parse_weights(const Architecture &a, const uint8_t *bytes, size_t len) {
  if (len < 4) throw Error(ILLUMINA_BAD_WEIGHTS, "weights: file is truncated");
  uint32_t hl = (uint32_t)bytes[0] | ((uint32_t)bytes[1] << 8) | ((uint32_t)bytes[2] << 16) |
                ((uint32_t)bytes[3] << 24);
  if (hl == 0 || 4 + (uint64_t)hl > len)
    throw Error(ILLUMINA_BAD_WEIGHTS, "weights: header length " + std::to_string(hl) + " does not fit the file");
  Json header;
  try {
    header = parse_json(std::string((const char *)bytes + 4, hl));
  } catch (const std::exception &e) {
    throw Error(ILLUMINA_BAD_WEIGHTS, std::string("weights: header is not valid JSON (") + e.what() + ")");
  }
  const Json *fmt = header.get("format");
  if (!fmt || fmt->type != Json::String || fmt->str != "idm/1")
    throw Error(ILLUMINA_BAD_WEIGHTS, "weights: unsupported format " + js_string_of(fmt) + ", expected idm/1");
  const Json *arch = header.get("arch");
  if (!arch || arch->type != Json::String || arch->str != a.name)
    throw Error(ILLUMINA_ARCH_MISMATCH, "weights: file is for " + js_string_of(arch) + ", this build is " + a.name);
  const Json *tensors = header.get("tensors");
  if (!tensors || tensors->type != Json::Object)
    throw Error(ILLUMINA_BAD_WEIGHTS, "weights: header has no tensors table");

  const size_t base = 4 + (size_t)hl;
  std::map<std::string, std::vector<float>> got;
  for (const auto &kv : tensors->obj) {
    const std::string &name = kv.first;
    const Json &info = kv.second;
    const Json *shape = info.get("shape"), *dtype = info.get("dtype"), *off = info.get("offset"),
               *length = info.get("length");
    if (!shape || shape->type != Json::Array || !off || off->type != Json::Number || !length ||
        length->type != Json::Number)
      throw Error(ILLUMINA_BAD_WEIGHTS, "weights: " + name + " has a malformed table entry");
    double count = 1;
    for (const auto &d : shape->arr) count *= d.num;
    bool f16 = dtype && dtype->type == Json::String && dtype->str == "f16";
    double nbytes = count * (f16 ? 2 : 4);
    if (length->num != nbytes)
      throw Error(ILLUMINA_BAD_WEIGHTS, "weights: " + name + " claims " + js_number(length->num) +
                                            " bytes but its shape needs " + js_number(nbytes));
    if (off->num < 0 || (double)base + off->num + nbytes > (double)len)
      throw Error(ILLUMINA_BAD_WEIGHTS, "weights: " + name + " extends past the end of the file");
    size_t n = (size_t)count, o = base + (size_t)off->num;
    std::vector<float> v(n);
    if (!f16) {
      std::memcpy(v.data(), bytes + o, n * 4);  // little-endian host
    } else {
      for (size_t i = 0; i < n; i++) {
        uint16_t h = (uint16_t)(bytes[o + 2 * i] | (bytes[o + 2 * i + 1] << 8));
        v[i] = (float)half_to_float(h);
      }
    }
    got[name] = std::move(v);
  }

  auto specs = weight_specs(a);
  std::vector<std::string> missing;
  std::vector<float> blob(weight_count(a));
  for (const auto &s : specs) {
    auto it = got.find(s.name);
    if (it == got.end()) {
      missing.push_back(s.name);
      continue;
    }
    if (it->second.size() != s.count) {
      std::string sh;
      for (size_t i = 0; i < s.shape.size(); i++) sh += (i ? ", " : "") + std::to_string(s.shape[i]);
      throw Error(ILLUMINA_BAD_WEIGHTS, "weights: " + s.name + " has " + std::to_string(it->second.size()) +
                                            " values, expected " + std::to_string(s.count) + " for shape [" + sh + "]");
    }
    std::memcpy(blob.data() + s.offset, it->second.data(), s.count * 4);
  }
  if (!missing.empty()) {
    std::string first;
    for (size_t i = 0; i < missing.size() && i < 5; i++) first += (i ? ", " : "") + missing[i];
    throw Error(ILLUMINA_BAD_WEIGHTS,
                "weights: " + std::to_string(missing.size()) + " tensor(s) missing, first few: " + first);
  }
  return blob;
}

std::vector<uint8_t> serialize_weights(const Architecture &a, const float *blob, size_t count) {
  auto specs = weight_specs(a);
  if (count != weight_count(a))
    throw Error(ILLUMINA_INVALID_ARG, "serializeWeights: blob has " + std::to_string(count) + " values, expected " +
                                          std::to_string(weight_count(a)));
  std::ostringstream h;
  h << "{\"format\":\"idm/1\",\"arch\":" << json_escape(a.name) << ",\"tensors\":{";
  size_t off = 0;
  for (size_t i = 0; i < specs.size(); i++) {
    const auto &s = specs[i];
    h << (i ? "," : "") << json_escape(s.name) << ":{\"dtype\":\"f32\",\"shape\":[";
    for (size_t d = 0; d < s.shape.size(); d++) h << (d ? "," : "") << s.shape[d];
    h << "],\"offset\":" << off << ",\"length\":" << s.count * 4 << "}";
    off += s.count * 4;
  }
  h << "}}";
  std::string header = h.str();
  std::vector<uint8_t> out(4 + header.size() + off);
  uint32_t hl = (uint32_t)header.size();
  out[0] = hl & 0xff, out[1] = (hl >> 8) & 0xff, out[2] = (hl >> 16) & 0xff, out[3] = (hl >> 24) & 0xff;
  std::memcpy(out.data() + 4, header.data(), header.size());
  std::memcpy(out.data() + 4 + header.size(), blob, count * 4);
  return out;
}

}  // namespace illumina
