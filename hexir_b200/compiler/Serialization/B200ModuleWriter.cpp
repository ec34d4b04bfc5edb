//===- B200ModuleWriter.cpp - host program -> .hxb for the B200 runtime ---===//
//
// Standard C++17 plus the C ABI of libhexir_b200 (link with -lhexir_b200).
//
//===----------------------------------------------------------------------===//
#include "B200ModuleWriter.h"

#include <map>
#include <memory>

#include "../Target/DeviceSpec.h"
#include "hexir_b200/hxb_writer.h"

namespace hexir_b200 {
namespace {

const char *placeableName(HostOpKind k) {
  switch (k) {
  case HostOpKind::Linear:
    return "hexir.linear";
  case HostOpKind::Add:
    return "hexir.add";
  case HostOpKind::Relu:
    return "hexir.relu";
  default:
    return nullptr;
  }
}

struct ProgramDeleter {
  void operator()(hexir_program_t *p) const { hexir_program_release(p); }
};

} // namespace

bool placementOf(const std::vector<HostOp> &ops, std::string *placement,
                 std::string *error) {
  std::map<std::string, std::string> byKind; // op name -> canonical device
  for (const HostOp &op : ops) {
    const char *name = placeableName(op.kind);
    if (!name)
      continue;
    const std::string dev =
        canonicalDeviceSpec(op.device.empty() ? "cpu" : op.device);
    if (dev.empty()) {
      *error = "'" + op.device + "' is not a device";
      return false;
    }
    auto it = byKind.emplace(name, dev).first;
    if (it->second != dev) {
      *error = std::string("ops of kind ") + name + " are placed on both '" +
               it->second + "' and '" + dev +
               "'; a module places each op kind on one device";
      return false;
    }
  }
  placement->clear();
  for (const auto &kv : byKind) {
    if (kv.second == "cpu")
      continue;
    if (!placement->empty())
      *placement += ",";
    *placement += kv.first + "=" + kv.second;
  }
  return true;
}

bool writeModule(const std::vector<HostOp> &ops, uint32_t flags,
                 std::string *bytes, std::string *error) {
  std::string placement;
  if (!placementOf(ops, &placement, error))
    return false;
  std::unique_ptr<hexir_program_t, ProgramDeleter> prog(hexir_program_create());
  if (!prog) {
    *error = "out of memory";
    return false;
  }
  hexir_program_t *p = prog.get();
  // Writer value of each op's result, by op index.
  std::vector<int32_t> value(ops.size(), -1);
  auto operand = [&](const HostOp &op, size_t i) -> int32_t {
    const int32_t src = op.operands.at(i);
    return src >= 0 && static_cast<size_t>(src) < ops.size() ? value[src] : -1;
  };
  for (size_t i = 0; i < ops.size(); ++i) {
    const HostOp &op = ops[i];
    int32_t v = -1;
    switch (op.kind) {
    case HostOpKind::BeginFunction:
      if (hexir_program_begin_function(p, op.name.c_str()) != HEXIR_OK) {
        *error = hexir_program_last_error(p);
        return false;
      }
      continue;
    case HostOpKind::Constant:
      if (op.data.size() != static_cast<size_t>(op.rows) * op.cols) {
        *error = "constant data does not match its shape";
        return false;
      }
      v = hexir_program_constant(p, op.data.data(), op.rows, op.cols);
      break;
    case HostOpKind::Splat:
      v = hexir_program_splat(p, op.splat, op.rows, op.cols);
      break;
    case HostOpKind::Linear:
      v = hexir_program_linear(p, operand(op, 0), operand(op, 1));
      break;
    case HostOpKind::Add:
      v = hexir_program_add(p, operand(op, 0), operand(op, 1));
      break;
    case HostOpKind::Relu:
      v = hexir_program_relu(p, operand(op, 0));
      break;
    case HostOpKind::Print:
      if (hexir_program_print(p, operand(op, 0)) != HEXIR_OK) {
        *error = hexir_program_last_error(p);
        return false;
      }
      continue;
    }
    if (v < 0) {
      *error = hexir_program_last_error(p);
      return false;
    }
    value[i] = v;
  }
  void *data = nullptr;
  size_t size = 0;
  if (hexir_program_emit_memory(p, placement.c_str(), flags, &data, &size) !=
      HEXIR_OK) {
    *error = hexir_program_last_error(p);
    return false;
  }
  bytes->assign(static_cast<const char *>(data), size);
  hexir_free(data);
  return true;
}

} // namespace hexir_b200
