// Layer table, cost model and weight specs of IlluminaDepth-448.
//
// build_architecture follows src/model/arch.ts:191-385 op for op (the op list,
// tensor names and channel widths are the reference's network definition and
// must be identical for .idm files and tensor names to interoperate);
// cost_of follows arch.ts:415-489; weight_specs follows
// src/model/weights.ts:29-63.
#include <sstream>

#include "host.h"

namespace illumina {

const char *op_kind_name(OpKind k) {
  switch (k) {
    case OpKind::Preprocess: return "preprocess";
    case OpKind::Conv: return "conv";
    case OpKind::Pw: return "pw";
    case OpKind::Dwpw: return "dwpw";
    case OpKind::Lateral: return "lateral";
    case OpKind::Head: return "head";
    case OpKind::BilateralUp: return "bilateralUp";
  }
  return "?";
}

const char *act_name(int act) {
  switch (act) {
    case ILLUMINA_ACT_RELU: return "relu";
    case ILLUMINA_ACT_RELU6: return "relu6";
    case ILLUMINA_ACT_HARDSWISH: return "hardswish";
    default: return "linear";
  }
}

const TensorShape &Architecture::shape(const std::string &n) const {
  auto it = tensors.find(n);
  if (it == tensors.end()) throw Error(ILLUMINA_INVALID_ARG, "unknown tensor " + n);
  return it->second;
}

namespace {

struct Builder {
  Architecture a;
  std::string T(const std::string &name, int h, int w, int c) {
    if (c % 4 != 0)
      throw Error(ILLUMINA_INVALID_ARG,
                  "tensor " + name + ": channel count " + std::to_string(c) + " is not a multiple of 4");
    if (!a.tensors.count(name)) a.tensor_order.push_back(name);
    a.tensors[name] = TensorShape{h, w, c};
    return name;
  }
  Op &push(OpKind kind, const std::string &name, const std::string &out) {
    Op op;
    op.kind = kind;
    op.name = name;
    op.out = out;
    a.ops.push_back(op);
    return a.ops.back();
  }
  // downBlock (arch.ts:242-265): dwpw s2 (linear -> hardswish) then pw project.
  std::string down_block(const std::string &p, const std::string &in, int h, int w, int expand, int out,
                         int k) {
    std::string mid = T(p + ".mid", h, w, expand);
    Op &d = push(OpKind::Dwpw, p + ".dw_expand", mid);
    d.in = in, d.k = k, d.stride = 2, d.mid_act = ILLUMINA_ACT_LINEAR, d.act = ILLUMINA_ACT_HARDSWISH;
    std::string o = T(p + ".out", h, w, out);
    Op &q = push(OpKind::Pw, p + ".project", o);
    q.in = mid, q.act = ILLUMINA_ACT_LINEAR;
    return o;
  }
  // irBlock (arch.ts:272-296): pw expand (hardswish) then dwpw + residual.
  std::string ir_block(const std::string &p, const std::string &in, int h, int w, int ch, int expand, int k) {
    std::string mid = T(p + ".mid", h, w, expand);
    Op &e = push(OpKind::Pw, p + ".expand", mid);
    e.in = in, e.act = ILLUMINA_ACT_HARDSWISH;
    std::string o = T(p + ".out", h, w, ch);
    Op &d = push(OpKind::Dwpw, p + ".dw_project", o);
    d.in = mid, d.k = k, d.stride = 1, d.mid_act = ILLUMINA_ACT_HARDSWISH, d.act = ILLUMINA_ACT_LINEAR;
    d.residual = in;
    return o;
  }
  // decoderLevel (arch.ts:335-360)
  std::string decoder(const std::string &p, const std::string &coarse, const std::string &skip, int h, int w,
                      int ch, int next) {
    std::string fused = T(p + ".fused", h, w, ch);
    Op &l = push(OpKind::Lateral, p + ".lateral", fused);
    l.coarse = coarse, l.skip = skip, l.act = ILLUMINA_ACT_LINEAR;
    std::string o = T(p + ".out", h, w, next);
    Op &d = push(OpKind::Dwpw, p + ".refine", o);
    d.in = fused, d.k = 3, d.stride = 1, d.mid_act = ILLUMINA_ACT_HARDSWISH, d.act = ILLUMINA_ACT_HARDSWISH;
    if (ch == next) d.residual = fused;
    return o;
  }
};

}  // namespace

Architecture build_architecture(int S) {
  if (S <= 0 || S % 32 != 0)
    throw Error(ILLUMINA_INVALID_ARG, "inputSize " + std::to_string(S) + " must be a multiple of 32");
  Builder b;
  auto r = [S](int level) { return S >> level; };
  std::string x0 = b.T("input", S, S, 4);
  b.push(OpKind::Preprocess, "preprocess", x0);
  std::string stem = b.T("stem", r(1), r(1), 16);
  {
    Op &o = b.push(OpKind::Conv, "stem", stem);
    o.in = x0, o.k = 3, o.stride = 2, o.act = ILLUMINA_ACT_HARDSWISH;
  }
  std::string s0 = b.T("s0", r(1), r(1), 24);
  {
    Op &o = b.push(OpKind::Dwpw, "e1", s0);
    o.in = stem, o.k = 3, o.stride = 1, o.mid_act = ILLUMINA_ACT_RELU6, o.act = ILLUMINA_ACT_LINEAR;
  }
  std::string t = b.down_block("e2", s0, r(2), r(2), 96, 32, 3);
  t = b.ir_block("e3", t, r(2), r(2), 32, 128, 3);
  std::string s1 = t;
  t = b.down_block("e4", s1, r(3), r(3), 128, 56, 5);
  t = b.ir_block("e5a", t, r(3), r(3), 56, 224, 5);
  t = b.ir_block("e5b", t, r(3), r(3), 56, 224, 5);
  std::string s2 = t;
  t = b.down_block("e6", s2, r(4), r(4), 224, 104, 5);
  t = b.ir_block("e7a", t, r(4), r(4), 104, 416, 5);
  t = b.ir_block("e7b", t, r(4), r(4), 104, 416, 5);
  t = b.ir_block("e7c", t, r(4), r(4), 104, 416, 5);
  std::string s3 = t;
  t = b.down_block("e8", s3, r(5), r(5), 416, 176, 5);
  t = b.ir_block("e9a", t, r(5), r(5), 176, 704, 5);
  t = b.ir_block("e9b", t, r(5), r(5), 176, 704, 5);
  t = b.ir_block("e9c", t, r(5), r(5), 176, 704, 5);
  std::string bottleneck = t;
  std::string d4 = b.T("d4", r(5), r(5), 96);
  {
    Op &o = b.push(OpKind::Pw, "d4.lateral", d4);
    o.in = bottleneck, o.act = ILLUMINA_ACT_HARDSWISH;
  }
  std::string d3 = b.decoder("d3", d4, s3, r(4), r(4), 96, 64);
  std::string d2 = b.decoder("d2", d3, s2, r(3), r(3), 64, 48);
  std::string d1 = b.decoder("d1", d2, s1, r(2), r(2), 48, 32);
  std::string d0 = b.decoder("d0", d1, s0, r(1), r(1), 32, 32);
  std::string low = b.T("depth_low", r(1), r(1), 4);
  {
    Op &o = b.push(OpKind::Head, "head", low);
    o.in = d0;
  }
  std::string full = b.T("depth", S, S, 4);
  {
    Op &o = b.push(OpKind::BilateralUp, "upsample", full);
    o.in = low;
  }
  b.a.name = "IlluminaDepth-448";
  b.a.input_size = S;
  const double mean[3] = {0.485, 0.456, 0.406}, stdv[3] = {0.229, 0.224, 0.225};
  for (int i = 0; i < 3; i++) b.a.mean[i] = mean[i], b.a.std[i] = stdv[i];
  return b.a;
}

std::vector<OpCost> cost_of(const Architecture &a, long *total_macs, long *total_params) {
  std::vector<OpCost> out;
  long tm = 0, tp = 0;
  for (const Op &op : a.ops) {
    OpCost c;
    c.name = op.name;
    c.kind = op.kind;
    const TensorShape &o = a.shape(op.out);
    switch (op.kind) {
      case OpKind::Conv: {
        const TensorShape &i = a.shape(op.in);
        c.macs = (long)o.h * o.w * o.c * i.c * op.k * op.k;
        c.params = (long)o.c * i.c * op.k * op.k + o.c;
        break;
      }
      case OpKind::Pw: {
        const TensorShape &i = a.shape(op.in);
        c.macs = (long)o.h * o.w * o.c * i.c;
        c.params = (long)o.c * i.c + o.c;
        break;
      }
      case OpKind::Dwpw: {
        const TensorShape &i = a.shape(op.in);
        c.macs = (long)o.h * o.w * i.c * op.k * op.k + (long)o.h * o.w * o.c * i.c;
        c.params = (long)i.c * op.k * op.k + i.c + (long)o.c * i.c + o.c;
        break;
      }
      case OpKind::Lateral: {
        const TensorShape &s = a.shape(op.skip);
        const TensorShape &cc = a.shape(op.coarse);
        if (cc.c != o.c)
          throw Error(ILLUMINA_INVALID_ARG, op.name + ": coarse tensor has " + std::to_string(cc.c) +
                                                " channels but the output has " + std::to_string(o.c));
        c.macs = (long)o.h * o.w * o.c * s.c;
        c.params = (long)o.c * s.c + o.c;
        break;
      }
      case OpKind::Head: {
        const TensorShape &i = a.shape(op.in);
        c.macs = (long)o.h * o.w * i.c;
        c.params = i.c + 1;
        break;
      }
      default: break;
    }
    tm += c.macs;
    tp += c.params;
    out.push_back(c);
  }
  if (total_macs) *total_macs = tm;
  if (total_params) *total_params = tp;
  return out;
}

std::vector<std::string> op_inputs(const Op &op) {
  switch (op.kind) {
    case OpKind::Preprocess: return {};
    case OpKind::Conv: return {op.in};
    case OpKind::Pw:
    case OpKind::Dwpw:
      if (!op.residual.empty()) return {op.in, op.residual};
      return {op.in};
    case OpKind::Lateral: return {op.coarse, op.skip};
    default: return {op.in};
  }
}

std::vector<WeightSpec> weight_specs(const Architecture &a) {
  std::vector<WeightSpec> out;
  size_t off = 0;
  auto add = [&](const std::string &n, std::vector<int> shape) {
    WeightSpec s;
    s.name = n;
    s.shape = shape;
    s.count = 1;
    for (int d : shape) s.count *= (size_t)d;
    s.offset = off;
    off += s.count;
    out.push_back(s);
  };
  auto c = [&](const std::string &n) { return a.shape(n).c; };
  for (const Op &op : a.ops) {
    switch (op.kind) {
      case OpKind::Conv:
        add(op.name + ".weight", {c(op.out), c(op.in), op.k, op.k});
        add(op.name + ".bias", {c(op.out)});
        break;
      case OpKind::Pw:
        add(op.name + ".weight", {c(op.out), c(op.in)});
        add(op.name + ".bias", {c(op.out)});
        break;
      case OpKind::Dwpw:
        add(op.name + ".dw_weight", {c(op.in), op.k, op.k});
        add(op.name + ".dw_bias", {c(op.in)});
        add(op.name + ".pw_weight", {c(op.out), c(op.in)});
        add(op.name + ".pw_bias", {c(op.out)});
        break;
      case OpKind::Lateral:
        add(op.name + ".weight", {c(op.out), c(op.skip)});
        add(op.name + ".bias", {c(op.out)});
        break;
      case OpKind::Head:
        add(op.name + ".weight", {1, c(op.in)});
        add(op.name + ".bias", {1});
        break;
      default: break;
    }
  }
  return out;
}

size_t weight_count(const Architecture &a) {
  size_t n = 0;
  for (const auto &s : weight_specs(a)) n += s.count;
  return n;
}

std::string json_escape(const std::string &s) {
  std::string o = "\"";
  for (char ch : s) {
    if (ch == '"' || ch == '\\') o += '\\', o += ch;
    else if ((unsigned char)ch < 0x20) {
      char buf[8];
      snprintf(buf, sizeof buf, "\\u%04x", ch);
      o += buf;
    } else o += ch;
  }
  return o + "\"";
}

std::string arch_to_json(const Architecture &a) {
  std::ostringstream js;
  js.precision(17);
  js << "{\"name\":" << json_escape(a.name) << ",\"inputSize\":" << a.input_size << ",\"mean\":[" << a.mean[0]
     << "," << a.mean[1] << "," << a.mean[2] << "],\"std\":[" << a.std[0] << "," << a.std[1] << ","
     << a.std[2] << "],\"tensors\":{";
  bool first = true;
  for (const auto &n : a.tensor_order) {
    const TensorShape &s = a.tensors.at(n);
    js << (first ? "" : ",") << json_escape(n) << ":[" << s.h << "," << s.w << "," << s.c << "]";
    first = false;
  }
  js << "},\"ops\":[";
  first = true;
  for (const Op &op : a.ops) {
    js << (first ? "" : ",") << "{\"kind\":" << json_escape(op_kind_name(op.kind))
       << ",\"name\":" << json_escape(op.name) << ",\"out\":" << json_escape(op.out);
    if (!op.in.empty()) js << ",\"in\":" << json_escape(op.in);
    if (op.kind == OpKind::Conv || op.kind == OpKind::Dwpw) js << ",\"k\":" << op.k << ",\"stride\":" << op.stride;
    if (op.kind == OpKind::Conv || op.kind == OpKind::Pw || op.kind == OpKind::Dwpw || op.kind == OpKind::Lateral)
      js << ",\"act\":" << json_escape(act_name(op.act));
    if (op.kind == OpKind::Dwpw) js << ",\"midAct\":" << json_escape(act_name(op.mid_act));
    if (!op.residual.empty()) js << ",\"residual\":" << json_escape(op.residual);
    if (!op.coarse.empty()) js << ",\"coarse\":" << json_escape(op.coarse) << ",\"skip\":" << json_escape(op.skip);
    js << "}";
    first = false;
  }
  long tm = 0, tp = 0;
  auto costs = cost_of(a, &tm, &tp);
  js << "],\"cost\":[";
  first = true;
  for (const auto &c : costs) {
    js << (first ? "" : ",") << "{\"name\":" << json_escape(c.name) << ",\"kind\":" << json_escape(op_kind_name(c.kind))
       << ",\"macs\":" << c.macs << ",\"params\":" << c.params << "}";
    first = false;
  }
  js << "],\"totalMacs\":" << tm << ",\"totalParams\":" << tp << ",\"specs\":[";
  first = true;
  for (const auto &s : weight_specs(a)) {
    js << (first ? "" : ",") << "[" << json_escape(s.name) << ",[";
    for (size_t i = 0; i < s.shape.size(); i++) js << (i ? "," : "") << s.shape[i];
    js << "]]";
    first = false;
  }
  js << "]}";
  return js.str();
}

}  // namespace illumina
