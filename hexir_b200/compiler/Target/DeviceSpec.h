//===- DeviceSpec.h - cpu | cuda | cuda:N | cuda:F-L -----------*- C++ -*-===//
//
// The placement grammar of the B200 runtime, for the reference compiler's
// -placement flag (tools/hexir/hexir.cpp:229-260), its target registry
// (compiler/Target/TargetInfo.cpp:15-18) and the `device` attribute the
// partition pass stamps (compiler/Dialect/Hexir/Transforms/Partition.cpp:
// 31-55).  The reference knows two devices, "cpu" and "cuda" ("gpu" is an
// alias); this adds a GPU ordinal, "cuda:N", and a row-sharded range of GPUs,
// "cuda:F-L" (the linear's rows split over GPUs F..L of one box).
//
// Standard C++ only, so it builds with or without LLVM: the same grammar as
// the runtime's .hxb writer (hexir_b200/csrc/writer/hxb_writer.cc,
// parse_device), which is what finally reads the stamped attribute.
//
//===----------------------------------------------------------------------===//
#ifndef HEXIR_B200_COMPILER_DEVICESPEC_H
#define HEXIR_B200_COMPILER_DEVICESPEC_H

#include <cstdint>
#include <string>
#include <string_view>

namespace hexir_b200 {

struct DeviceSpec {
  bool cuda = false;    // false: the host
  uint32_t first = 0;   // first GPU ordinal
  uint32_t count = 1;   // GPUs the rows are split over (1: not sharded)
  bool ordinal = false; // written with an explicit ":N" / ":F-L"
};

// Parses "cpu", "cuda", "gpu", "cuda:N", "cuda:F-L", "gpu:N", "gpu:F-L"
// (N, F, L decimal, at most 4 digits, F <= L).  False for anything else.
bool parseDeviceSpec(std::string_view text, DeviceSpec *out);

// The device kind the target registry checks support against: "cpu" or
// "cuda" (every GPU spec), or "" for text that is not a device.
std::string_view deviceKind(std::string_view text);

// The canonical spelling stamped into `device` attributes: "cpu", "cuda",
// "cuda:N", "cuda:F-L" ("gpu" spelled "cuda", leading zeros dropped, and
// "cuda:F-F" spelled "cuda:F").  "" for text that is not a device.
std::string canonicalDeviceSpec(std::string_view text);

// True for every spec whose kind is "cuda".  The compiler's passes that
// select GPU work (HexirToTIR, HexTIRToGPU, CudaToGpu, the serializer)
// compare with this instead of `== "cuda"`, so an ordinal passes through.
bool isCudaSpec(std::string_view text);

} // namespace hexir_b200

#endif // HEXIR_B200_COMPILER_DEVICESPEC_H
