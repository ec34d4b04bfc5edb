// hxb_writer.cc -- program builder and .hxb serializer
// (include/hexir_b200/hxb_writer.h).
//
// Serialization follows the reference serializer's observable output
// (compiler/Serialization/ModuleSerializer.cpp:47-425): byte layout, splat
// expansion, 8-byte padding, module-wide slot numbering in op order, CONST
// before use, ALLOC + DISPATCH per compute op with the destination last,
// PRINT, END per function.  Executable naming and kinds follow
// compiler/Conversion/HexirToTIR/HexirToTIR.cpp:251-281; placement parsing
// follows tools/hexir/hexir.cpp:229-260 with compiler/Target/TargetInfo.cpp.

#include "hexir_b200/hxb_writer.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

#include "hexir_b200/kernels.h"
#include "hexir_runtime/module.h"
#include "hexir_runtime/program.h"

namespace {

enum class OpKind { Constant, Linear, Add, Relu, Activation, Print };

// The activations the dialect declares (HexirOps.td:189-308), by the kernel
// kind that runs them.
struct ActivationName {
  const char *name;
  uint32_t kind;
};
const ActivationName kActivations[] = {
    {"leaky_relu", HEXIR_KERNEL_LEAKY_RELU}, {"elu", HEXIR_KERNEL_ELU},
    {"sigmoid", HEXIR_KERNEL_SIGMOID},       {"tanh", HEXIR_KERNEL_TANH},
    {"softmax", HEXIR_KERNEL_SOFTMAX},       {"gelu", HEXIR_KERNEL_GELU},
    {"swish", HEXIR_KERNEL_SWISH},           {"mish", HEXIR_KERNEL_MISH},
};

const char *activation_name(uint32_t kind) {
  for (const ActivationName &a : kActivations)
    if (a.kind == kind)
      return a.name;
  return "";
}

struct Value {
  uint32_t rows = 0, cols = 0;
  int def = -1;   // defining op
  int uses = 0;
  int func = -1;
};

struct Op {
  OpKind kind;
  std::vector<int> operands;
  int result = -1;
  std::vector<double> data;  // constants
  bool splat = false;
  double splat_value = 0.0;
  uint32_t act = 0;  // Activation: its kernel kind
};

struct Function {
  std::string name;
  std::vector<int> ops;
};

struct DeviceSpec {
  bool cuda = false;
  uint32_t first = 0, count = 1;
  bool operator==(const DeviceSpec &o) const {
    return cuda == o.cuda && (!cuda || (first == o.first && count == o.count));
  }
};

// Little-endian byte buffer with the reference serializer's padding rule.
struct Bytes {
  std::vector<char> b;
  void raw(const void *p, size_t n) {
    const char *c = static_cast<const char *>(p);
    b.insert(b.end(), c, c + n);
  }
  void u32(uint32_t v) { raw(&v, 4); }
  void u64(uint64_t v) { raw(&v, 8); }
  void pad_to(size_t a) {
    while (b.size() % a)
      b.push_back(0);
  }
  size_t size() const { return b.size(); }
};

const char *op_name(const Op &op) {
  switch (op.kind) {
  case OpKind::Linear: return "linear";
  case OpKind::Add: return "add";
  case OpKind::Relu: return "relu";
  case OpKind::Activation: return activation_name(op.act);
  default: return "";
  }
}

bool is_compute(OpKind k) {
  return k == OpKind::Linear || k == OpKind::Add || k == OpKind::Relu ||
         k == OpKind::Activation;
}

void write_name(char (&dst)[HEXIR_NAME_SIZE], const std::string &name) {
  std::memset(dst, 0, HEXIR_NAME_SIZE);
  std::memcpy(dst, name.data(), std::min<size_t>(name.size(), HEXIR_NAME_SIZE - 1));
}

// "cpu" | "cuda" | "gpu" | "cuda:N" | "cuda:F-L" ("gpu:" likewise).
bool parse_device(const std::string &text, DeviceSpec *out) {
  if (text == "cpu") {
    *out = DeviceSpec{};
    return true;
  }
  std::string rest;
  if (text == "cuda" || text == "gpu") {
    *out = DeviceSpec{true, 0, 1};
    return true;
  }
  if (text.rfind("cuda:", 0) == 0)
    rest = text.substr(5);
  else if (text.rfind("gpu:", 0) == 0)
    rest = text.substr(4);
  else
    return false;
  auto number = [](const std::string &s, uint32_t *v) {
    if (s.empty() || s.size() > 4)
      return false;
    for (char c : s)
      if (c < '0' || c > '9')
        return false;
    *v = static_cast<uint32_t>(std::stoul(s));
    return true;
  };
  size_t dash = rest.find('-');
  uint32_t first = 0, last = 0;
  if (dash == std::string::npos) {
    if (!number(rest, &first))
      return false;
    *out = DeviceSpec{true, first, 1};
    return true;
  }
  if (!number(rest.substr(0, dash), &first) ||
      !number(rest.substr(dash + 1), &last) || last < first)
    return false;
  *out = DeviceSpec{true, first, last - first + 1};
  return true;
}

}  // namespace

struct hexir_program_t {
  std::vector<Value> values;
  std::vector<Op> ops;
  std::vector<Function> funcs;
  std::string error;

  Function &current() {
    if (funcs.empty())
      funcs.push_back(Function{"main", {}});
    return funcs.back();
  }

  int add_op(Op op, uint32_t rows, uint32_t cols) {
    Function &f = current();
    const int fi = static_cast<int>(funcs.size()) - 1;
    for (int v : op.operands) {
      if (v < 0 || v >= static_cast<int>(values.size()) || values[v].func != fi) {
        error = "operand is not a value of this function";
        return -1;
      }
    }
    for (int v : op.operands)
      values[v].uses++;
    const int index = static_cast<int>(ops.size());
    if (op.kind != OpKind::Print) {
      Value val;
      val.rows = rows;
      val.cols = cols;
      val.def = index;
      val.func = fi;
      op.result = static_cast<int>(values.size());
      values.push_back(val);
    }
    ops.push_back(std::move(op));
    f.ops.push_back(index);
    return ops.back().result;
  }

  bool valid(int v) const { return v >= 0 && v < static_cast<int>(values.size()); }

  hexir_status_t emit(const char *placement, uint32_t flags, Bytes *out);
};

namespace {

// The placeable ops are the reference's three (compiler/Target/
// TargetInfo.cpp:21-23), plus the activations when they are being written.
hexir_status_t parse_placement(const char *text,
                               std::map<std::string, DeviceSpec> *spec,
                               std::string *error, bool activations) {
  (*spec)["hexir.linear"] = DeviceSpec{};
  (*spec)["hexir.add"] = DeviceSpec{};
  (*spec)["hexir.relu"] = DeviceSpec{};
  if (activations)
    for (const ActivationName &a : kActivations)
      (*spec)[std::string("hexir.") + a.name] = DeviceSpec{};
  if (!text || !*text)
    return HEXIR_OK;
  std::string all(text);
  size_t pos = 0;
  while (pos <= all.size()) {
    size_t comma = all.find(',', pos);
    std::string entry = all.substr(pos, comma == std::string::npos
                                            ? std::string::npos
                                            : comma - pos);
    pos = comma == std::string::npos ? all.size() + 1 : comma + 1;
    size_t eq = entry.find('=');
    std::string op = eq == std::string::npos ? entry : entry.substr(0, eq);
    std::string dev = eq == std::string::npos ? "" : entry.substr(eq + 1);
    if (op.empty() || dev.empty()) {
      *error = "error: -placement entry '" + entry +
               "' is not of the form <op-name>=<device>";
      return HEXIR_ERROR_INVALID_ARGUMENT;
    }
    DeviceSpec d;
    if (!parse_device(dev, &d)) {
      *error = "error: '" + dev +
               "' is not a device; expected cpu, cuda or gpu";
      return HEXIR_ERROR_INVALID_ARGUMENT;
    }
    if (!spec->count(op)) {
      *error = "error: '" + op + "' is not a placeable op";
      return HEXIR_ERROR_INVALID_ARGUMENT;
    }
    (*spec)[op] = d;
  }
  return HEXIR_OK;
}

std::string op_key(const Op &op) {
  return std::string("hexir.") + op_name(op);
}

}  // namespace

hexir_status_t hexir_program_t::emit(const char *placement, uint32_t flags,
                                     Bytes *out) {
  std::map<std::string, DeviceSpec> spec;
  hexir_status_t st = parse_placement(placement, &spec, &error,
                                      (flags & HEXIR_EMIT_ACTIVATIONS) != 0);
  if (st != HEXIR_OK)
    return st;
  // The reference serializer has no kernel for the activations and refuses
  // them (ModuleSerializer.cpp:368); they are written only on request.
  if (!(flags & HEXIR_EMIT_ACTIVATIONS))
    for (const Op &op : ops)
      if (op.kind == OpKind::Activation) {
        error = "'" + op_key(op) +
                "' op cannot serialize this op into a host program";
        return HEXIR_ERROR_UNIMPLEMENTED;
      }

  // Kernel names in walk order (functions in order, ops in order), every
  // compute op taking a number even if fusion later folds it away.
  std::vector<std::string> kernel_name(ops.size());
  std::vector<DeviceSpec> where(ops.size());
  unsigned counter = 0;
  for (const Function &f : funcs)
    for (int oi : f.ops)
      if (is_compute(ops[oi].kind)) {
        kernel_name[oi] = std::string(op_name(ops[oi])) + "_" +
                          std::to_string(counter++);
        where[oi] = spec.count(op_key(ops[oi])) ? spec[op_key(ops[oi])]
                                                : DeviceSpec{};
      }

  // Fusions on a GPU, each where the intermediate value has no other user and
  // every op sits on the same device spec:
  //   linear -> add [-> relu]  one matmul_add[_relu] executable, named after
  //                            the linear, dispatched where the add stands
  //                            (its addend may be computed after the linear);
  //   linear -> relu           one matmul_relu, dispatched where the linear
  //                            stands.
  std::vector<bool> fused(ops.size(), false), folded(ops.size(), false);
  std::vector<uint32_t> fused_kind(ops.size(), 0);  // linear op -> kind
  std::vector<int> add_linear(ops.size(), -1);  // add op -> its linear op
  std::vector<int> addend_of(ops.size(), -1);   // add op -> addend value
  std::vector<int> alias(values.size(), -1);    // folded result -> kept result
  auto fusable = [&](int value, int user_op) {
    const int def = values[value].def;
    return def >= 0 && ops[def].kind == OpKind::Linear && values[value].uses == 1 &&
           !fused[def] && where[user_op].cuda && where[user_op] == where[def];
  };
  if (!(flags & HEXIR_EMIT_NO_FUSE)) {
    for (size_t oi = 0; oi < ops.size(); ++oi) {
      const Op &add = ops[oi];
      if (add.kind != OpKind::Add)
        continue;
      for (int i = 0; i < 2; ++i) {
        const int in = add.operands[i];
        if (!fusable(in, static_cast<int>(oi)))
          continue;
        const int def = values[in].def;
        fused[def] = true;
        fused_kind[def] = HEXIR_KERNEL_MATMUL_ADD;
        add_linear[oi] = def;
        addend_of[oi] = add.operands[1 - i];
        break;
      }
    }
    for (size_t oi = 0; oi < ops.size(); ++oi) {
      const Op &r = ops[oi];
      if (r.kind != OpKind::Relu)
        continue;
      const int in = r.operands[0];
      const int def = values[in].def;
      if (def < 0 || values[in].uses != 1 || !where[oi].cuda ||
          !(where[oi] == where[def]))
        continue;
      if (ops[def].kind == OpKind::Add && add_linear[def] >= 0) {
        fused_kind[add_linear[def]] = HEXIR_KERNEL_MATMUL_ADD_RELU;
        folded[oi] = true;
        alias[r.result] = in;
      } else if (ops[def].kind == OpKind::Linear && !fused[def]) {
        fused[def] = true;
        fused_kind[def] = HEXIR_KERNEL_MATMUL_RELU;
        folded[oi] = true;
        alias[r.result] = in;
      }
    }
  }
  // The op whose position carries op oi's dispatch, and the op whose
  // executable it runs.
  auto deferred = [&](int oi) {
    return ops[oi].kind == OpKind::Linear && fused[oi] &&
           fused_kind[oi] != HEXIR_KERNEL_MATMUL_RELU;
  };

  const void *image = nullptr;
  size_t image_size = 0;
  const bool images = !(flags & HEXIR_EMIT_NO_IMAGE);

  // EXECUTABLES, in walk order.
  std::vector<hexir_executable_entry_t> entries;
  std::vector<hexir_launch_entry_t> launch;
  std::map<int, uint32_t> exe_index;  // op -> executable index
  bool any_library = false;
  for (const Function &f : funcs) {
    for (int at : f.ops) {
      if (!is_compute(ops[at].kind) || folded[at] || deferred(at))
        continue;
      // A fused add carries its linear's executable.
      const int oi = add_linear[at] >= 0 ? add_linear[at] : at;
      const Op &op = ops[oi];
      hexir_executable_entry_t e;
      std::memset(&e, 0, sizeof(e));
      write_name(e.name, kernel_name[oi]);
      const Value &dst = values[ops[at].result];
      if (op.kind == OpKind::Linear)
        e.kind = fused[oi] ? fused_kind[oi]
                           : static_cast<uint32_t>(HEXIR_KERNEL_MATMUL);
      else if (op.kind == OpKind::Activation)
        e.kind = op.act;
      else
        e.kind = op.kind == OpKind::Add ? HEXIR_KERNEL_ADD : HEXIR_KERNEL_RELU;
      e.device = where[oi].cuda ? 1u : 0u;
      e.m = dst.rows;
      e.n = dst.cols;
      if (op.kind == OpKind::Linear)
        e.k = values[op.operands[0]].cols;
      e.elem_size = 8;
      hexir_launch_entry_t l;
      std::memset(&l, 0, sizeof(l));
      if (where[oi].cuda && images) {
        if (!image) {
          hexir_cuda_kernel_image(&image, &image_size);
          if (!image || !image_size) {
            error = "no sm_100a kernel image is embedded in this library";
            return HEXIR_ERROR_UNIMPLEMENTED;
          }
        }
        e.image_offset = 0;  // fixed up below: all entries share one image
        e.image_size = static_cast<uint32_t>(image_size);
        if (op.kind == OpKind::Linear) {
          e.grid_x = ((e.m + 127) / 128) * ((e.n + 127) / 128);
          e.grid_y = 1;
        } else {
          const uint64_t pairs = (static_cast<uint64_t>(e.m) * e.n + 1) / 2;
          e.grid_x = static_cast<uint32_t>(std::max<uint64_t>(
              1, std::min<uint64_t>((pairs + 1023) / 1024, 148 * 8)));
          e.grid_y = 1;
        }
        e.block_x = 256;
        e.block_y = 1;
        l.abi = HEXIR_LAUNCH_ABI_V1;
        l.flags = HEXIR_LAUNCH_FLAG_LIBRARY;
        l.device_first = where[oi].first;
        l.device_count = where[oi].count;
        any_library = true;
      }
      exe_index[at] = static_cast<uint32_t>(entries.size());
      entries.push_back(e);
      launch.push_back(l);
    }
  }
  Bytes executables;
  {
    uint32_t base = static_cast<uint32_t>(sizeof(hexir_executable_header_t) +
                                          entries.size() *
                                              sizeof(hexir_executable_entry_t));
    base += (8 - (base % 8)) % 8;
    hexir_executable_header_t header{static_cast<uint32_t>(entries.size()), 0};
    executables.raw(&header, sizeof(header));
    for (hexir_executable_entry_t &e : entries) {
      if (e.image_size)
        e.image_offset = base;
      executables.raw(&e, sizeof(e));
    }
    executables.pad_to(8);
    if (image && any_library)
      executables.raw(image, image_size);
  }

  // SYMBOLS, PROGRAM, RODATA.
  Bytes symbols, program, rodata;
  std::vector<int64_t> slot_of(values.size(), -1);
  uint64_t next_slot = 0;
  auto command = [&](uint32_t kind, std::initializer_list<uint64_t> operands) {
    program.u32(kind);
    program.u32(static_cast<uint32_t>(operands.size()));
    for (uint64_t o : operands)
      program.u64(o);
  };
  for (const Function &f : funcs) {
    hexir_symbol_entry_t sym;
    std::memset(&sym, 0, sizeof(sym));
    write_name(sym.name, f.name);
    sym.program_offset = static_cast<uint32_t>(program.size());
    symbols.raw(&sym, sizeof(sym));
    for (int oi : f.ops) {
      const Op &op = ops[oi];
      if (op.kind == OpKind::Constant) {
        const Value &v = values[op.result];
        if (v.uses == 0)
          continue;  // constants with no users never reach the runtime
        const uint64_t offset = rodata.size();
        const uint64_t bytes = static_cast<uint64_t>(v.rows) * v.cols * 8;
        if (op.splat) {
          for (uint64_t w = 0; w < bytes; w += 8)
            rodata.raw(&op.splat_value, 8);
        } else {
          rodata.raw(op.data.data(), op.data.size() * 8);
        }
        rodata.pad_to(8);
        slot_of[op.result] = static_cast<int64_t>(next_slot++);
        command(HEXIR_CMD_CONST, {static_cast<uint64_t>(slot_of[op.result]),
                                  offset, bytes});
        continue;
      }
      if (is_compute(op.kind)) {
        if (folded[oi]) {
          slot_of[op.result] = slot_of[alias[op.result]];
          continue;
        }
        if (deferred(oi))
          continue;  // dispatched where its add stands
        // Operands: the op's own, or for a fused add its linear's and then
        // the addend.
        std::vector<int> operands = op.operands;
        if (add_linear[oi] >= 0) {
          operands = ops[add_linear[oi]].operands;
          operands.push_back(addend_of[oi]);
        }
        const Value &dst = values[op.result];
        const uint64_t d = next_slot++;
        slot_of[op.result] = static_cast<int64_t>(d);
        command(HEXIR_CMD_ALLOC, {d, static_cast<uint64_t>(dst.rows) * dst.cols * 8});
        program.u32(HEXIR_CMD_DISPATCH);
        program.u32(static_cast<uint32_t>(2 + operands.size() + 1));
        program.u64(exe_index[oi]);
        program.u64(operands.size() + 1);
        for (int a : operands) {
          if (slot_of[a] < 0) {
            error = "argument has no slot; it is not produced by a constant or "
                    "a call in this function";
            return HEXIR_ERROR_INVALID_ARGUMENT;
          }
          program.u64(static_cast<uint64_t>(slot_of[a]));
        }
        program.u64(d);
        continue;
      }
      // print
      const int v = op.operands[0];
      if (slot_of[v] < 0) {
        error = "operand has no slot";
        return HEXIR_ERROR_INVALID_ARGUMENT;
      }
      command(HEXIR_CMD_PRINT, {static_cast<uint64_t>(slot_of[v]), values[v].rows,
                                values[v].cols});
    }
    command(HEXIR_CMD_END, {});
  }

  Bytes launch_section;
  if (any_library) {
    hexir_launch_header_t header{static_cast<uint32_t>(launch.size()), 0};
    launch_section.raw(&header, sizeof(header));
    for (const hexir_launch_entry_t &l : launch)
      launch_section.raw(&l, sizeof(l));
  }

  struct Section {
    uint32_t kind;
    const Bytes *data;
  };
  std::vector<Section> sections = {{HEXIR_SECTION_SYMBOLS, &symbols},
                                   {HEXIR_SECTION_PROGRAM, &program},
                                   {HEXIR_SECTION_RODATA, &rodata},
                                   {HEXIR_SECTION_EXECUTABLES, &executables}};
  if (any_library)
    sections.push_back({HEXIR_SECTION_LAUNCH, &launch_section});

  hexir_module_header_t header;
  std::memset(&header, 0, sizeof(header));
  std::memcpy(header.magic, HEXIR_MODULE_MAGIC, HEXIR_MODULE_MAGIC_SIZE);
  header.version = HEXIR_MODULE_VERSION;
  header.section_count = static_cast<uint32_t>(sections.size());
  out->raw(&header, sizeof(header));
  uint64_t offset = sizeof(hexir_module_header_t) +
                    sections.size() * sizeof(hexir_section_entry_t);
  for (const Section &s : sections) {
    offset += (8 - (offset % 8)) % 8;
    hexir_section_entry_t e;
    std::memset(&e, 0, sizeof(e));
    e.kind = s.kind;
    e.offset = offset;
    e.size = s.data->size();
    out->raw(&e, sizeof(e));
    offset += s.data->size();
  }
  for (const Section &s : sections) {
    out->pad_to(8);
    out->raw(s.data->b.data(), s.data->size());
  }
  return HEXIR_OK;
}

extern "C" {

hexir_program_t *hexir_program_create(void) {
  return new (std::nothrow) hexir_program_t;
}

void hexir_program_release(hexir_program_t *program) { delete program; }

hexir_status_t hexir_program_begin_function(hexir_program_t *p,
                                            const char *name) {
  if (!p || !name || !*name)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  p->funcs.push_back(Function{name, {}});
  return HEXIR_OK;
}

int32_t hexir_program_constant(hexir_program_t *p, const double *data,
                               uint32_t rows, uint32_t cols) {
  if (!p || (!data && rows && cols))
    return -1;
  try {
    Op op{OpKind::Constant, {}, -1, {}, false, 0.0};
    op.data.assign(data, data + static_cast<size_t>(rows) * cols);
    return p->add_op(std::move(op), rows, cols);
  } catch (const std::bad_alloc &) {
    p->error = "out of host memory for a constant";
    return -1;
  }
}

int32_t hexir_program_splat(hexir_program_t *p, double value, uint32_t rows,
                            uint32_t cols) {
  if (!p)
    return -1;
  Op op{OpKind::Constant, {}, -1, {}, true, value};
  return p->add_op(std::move(op), rows, cols);
}

int32_t hexir_program_linear(hexir_program_t *p, int32_t input, int32_t weight) {
  if (!p)
    return -1;
  if (!p->valid(input) || !p->valid(weight)) {
    p->error = "hexir.linear: unknown operand";
    return -1;
  }
  const Value &a = p->values[input], &w = p->values[weight];
  if (a.cols != w.rows) {
    p->error = "hexir.linear: input is " + std::to_string(a.rows) + "x" +
               std::to_string(a.cols) + " but weight is " +
               std::to_string(w.rows) + "x" + std::to_string(w.cols);
    return -1;
  }
  return p->add_op(Op{OpKind::Linear, {input, weight}, -1, {}, false, 0.0},
                   a.rows, w.cols);
}

int32_t hexir_program_add(hexir_program_t *p, int32_t lhs, int32_t rhs) {
  if (!p)
    return -1;
  if (!p->valid(lhs) || !p->valid(rhs)) {
    p->error = "hexir.add: unknown operand";
    return -1;
  }
  const Value &a = p->values[lhs], &b = p->values[rhs];
  if (a.rows != b.rows || a.cols != b.cols) {
    p->error = "hexir.add: operand shapes differ";
    return -1;
  }
  return p->add_op(Op{OpKind::Add, {lhs, rhs}, -1, {}, false, 0.0}, a.rows,
                   a.cols);
}

int32_t hexir_program_relu(hexir_program_t *p, int32_t input) {
  if (!p)
    return -1;
  if (!p->valid(input)) {
    p->error = "hexir.relu: unknown operand";
    return -1;
  }
  const Value &a = p->values[input];
  return p->add_op(Op{OpKind::Relu, {input}, -1, {}, false, 0.0}, a.rows,
                   a.cols);
}

int32_t hexir_program_activation(hexir_program_t *p, const char *op,
                                 int32_t input) {
  if (!p)
    return -1;
  std::string name = op ? op : "";
  if (name.rfind("hexir.", 0) == 0)
    name = name.substr(6);
  uint32_t kind = 0;
  for (const ActivationName &a : kActivations)
    if (name == a.name)
      kind = a.kind;
  if (!kind) {
    p->error = "'" + name + "' is not an activation";
    return -1;
  }
  if (!p->valid(input)) {
    p->error = "hexir." + name + ": unknown operand";
    return -1;
  }
  const Value &a = p->values[input];
  Op o{OpKind::Activation, {input}, -1, {}, false, 0.0};
  o.act = kind;
  return p->add_op(o, a.rows, a.cols);
}

hexir_status_t hexir_program_print(hexir_program_t *p, int32_t value) {
  if (!p)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  if (!p->valid(value)) {
    p->error = "hexir.print: unknown operand";
    return HEXIR_ERROR_INVALID_ARGUMENT;
  }
  p->error.clear();
  p->add_op(Op{OpKind::Print, {value}, -1, {}, false, 0.0}, 0, 0);
  return p->error.empty() ? HEXIR_OK : HEXIR_ERROR_INVALID_ARGUMENT;
}

hexir_status_t hexir_program_emit_memory(hexir_program_t *p,
                                         const char *placement, uint32_t flags,
                                         void **data, size_t *size) {
  if (!p || !data || !size)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *data = nullptr;
  *size = 0;
  Bytes out;
  hexir_status_t st;
  try {
    st = p->emit(placement, flags, &out);
  } catch (const std::bad_alloc &) {
    p->error = "out of host memory while serializing";
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  if (st != HEXIR_OK)
    return st;
  void *buf = std::malloc(out.size() ? out.size() : 1);
  if (!buf)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  std::memcpy(buf, out.b.data(), out.size());
  *data = buf;
  *size = out.size();
  return HEXIR_OK;
}

hexir_status_t hexir_program_emit_file(hexir_program_t *p, const char *placement,
                                       uint32_t flags, const char *path) {
  if (!p || !path)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  Bytes out;
  hexir_status_t st;
  try {
    st = p->emit(placement, flags, &out);
  } catch (const std::bad_alloc &) {
    p->error = "out of host memory while serializing";
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  if (st != HEXIR_OK)
    return st;
  FILE *f = std::fopen(path, "wb");
  if (!f) {
    p->error = std::string("cannot open ") + path + " for writing";
    return HEXIR_ERROR_IO;
  }
  const size_t wrote = std::fwrite(out.b.data(), 1, out.size(), f);
  const int closed = std::fclose(f);
  if (wrote != out.size() || closed != 0) {
    p->error = std::string("short write to ") + path;
    return HEXIR_ERROR_IO;
  }
  return HEXIR_OK;
}

void hexir_free(void *data) { std::free(data); }

const char *hexir_program_last_error(const hexir_program_t *p) {
  return p ? p->error.c_str() : "null program";
}

void hexir_rng_seed(hexir_rng_t *rng, uint64_t seed) {
  if (rng)
    rng->state = seed;
}

static inline uint64_t splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline double unit_double(uint64_t *state) {
  return static_cast<double>(splitmix64(state) >> 11) * 0x1.0p-53;
}

void hexir_rng_uniform(hexir_rng_t *rng, double *out, size_t n, double lo,
                       double hi) {
  if (!rng || !out)
    return;
  const double span = hi - lo;
  for (size_t i = 0; i < n; ++i)
    out[i] = lo + span * unit_double(&rng->state);
}

void hexir_rng_normal(hexir_rng_t *rng, double *out, size_t n, double mean,
                      double stddev) {
  if (!rng || !out)
    return;
  const double two_pi = 6.283185307179586476925286766559;
  for (size_t i = 0; i < n; ++i) {
    const double u1 = unit_double(&rng->state);
    const double u2 = unit_double(&rng->state);
    out[i] = mean + stddev * std::sqrt(-2.0 * std::log(1.0 - u1)) *
                        std::cos(two_pi * u2);
  }
}

}  // extern "C"
