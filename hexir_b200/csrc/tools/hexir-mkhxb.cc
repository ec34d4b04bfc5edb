// hexir-mkhxb -- write a .hxb module from a textual hexir program.
//
// Stands in for `hexir -emit=hxb` (tools/hexir/hexir.cpp:125-176,512), whose
// MLIR/LLVM dependency does not build here, with the same flags for this
// path:
//
//   hexir-mkhxb [-emit=hxb] [-o out.hxb] [-placement=op=dev[,...]] [input.mlir]
//
// With no input it writes the built-in program of the reference compiler
// (compiler/Support/Builder.cpp:264-327: [[3,1],[2,2]] . [[1,5],[5,2]],
// printed).  Additions: --no-fuse keeps linear and relu as two executables;
// --no-image writes cuda-placed executables as descriptors only;
// --activations writes the dialect's activations (leaky_relu ... mish) as
// kernel kinds 7-14 instead of refusing them; placement devices cuda:N and
// cuda:F-L.

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>

#include "hexir_b200/hxb_writer.h"

static int usage() {
  std::fprintf(stderr,
               "usage: hexir-mkhxb [-emit=hxb] [-o <file>] "
               "[-placement=<op>=<device>[,...]]\n"
               "                   [--no-fuse] [--no-image] [--activations] "
               "[input.mlir]\n"
               "devices: cpu, cuda, gpu, cuda:N, cuda:F-L (rows split over "
               "GPUs F..L)\n"
               "placeable ops: hexir.add, hexir.linear, hexir.relu; with "
               "--activations also\n"
               "  hexir.leaky_relu, hexir.elu, hexir.sigmoid, hexir.tanh, "
               "hexir.softmax,\n"
               "  hexir.gelu, hexir.swish, hexir.mish\n");
  return 2;
}

static hexir_program_t *builtin_program() {
  hexir_program_t *p = hexir_program_create();
  const double unused[2] = {3.0, 1.0};
  const double a[4] = {3.0, 1.0, 2.0, 2.0};
  const double b[4] = {1.0, 5.0, 5.0, 2.0};
  hexir_program_constant(p, unused, 1, 2);  // no users: dropped on emit
  int ca = hexir_program_constant(p, a, 2, 2);
  int cb = hexir_program_constant(p, b, 2, 2);
  int lin = hexir_program_linear(p, ca, cb);
  hexir_program_print(p, lin);
  return p;
}

int main(int argc, char **argv) {
  std::string out = "out.hxb", placement, input;
  uint32_t flags = 0;
  for (int i = 1; i < argc; ++i) {
    std::string arg = argv[i];
    if (arg == "-o" && i + 1 < argc) {
      out = argv[++i];
    } else if (arg.rfind("-o=", 0) == 0) {
      out = arg.substr(3);
    } else if (arg.rfind("-placement=", 0) == 0 ||
               arg.rfind("--placement=", 0) == 0) {
      std::string v = arg.substr(arg.find('=') + 1);
      placement += (placement.empty() ? "" : ",") + v;
    } else if (arg == "-emit=hxb" || arg == "--emit=hxb") {
    } else if (arg.rfind("-emit=", 0) == 0) {
      std::fprintf(stderr, "hexir-mkhxb: only -emit=hxb is supported\n");
      return 2;
    } else if (arg == "--no-fuse") {
      flags |= HEXIR_EMIT_NO_FUSE;
    } else if (arg == "--no-image") {
      flags |= HEXIR_EMIT_NO_IMAGE;
    } else if (arg == "--activations") {
      flags |= HEXIR_EMIT_ACTIVATIONS;
    } else if (arg == "-h" || arg == "--help") {
      return usage();
    } else if (!arg.empty() && arg[0] == '-' && arg != "-") {
      return usage();
    } else {
      input = arg;
    }
  }

  hexir_program_t *program = nullptr;
  if (input.empty()) {
    program = builtin_program();
  } else {
    std::string text;
    if (input == "-") {
      std::stringstream ss;
      ss << std::cin.rdbuf();
      text = ss.str();
    } else {
      std::ifstream f(input);
      if (!f) {
        std::fprintf(stderr, "hexir-mkhxb: cannot read '%s'\n", input.c_str());
        return 1;
      }
      std::stringstream ss;
      ss << f.rdbuf();
      text = ss.str();
    }
    char error[512] = {0};
    if (hexir_program_parse(text.c_str(), &program, error, sizeof(error)) !=
        HEXIR_OK) {
      std::fprintf(stderr, "%s:%s\n", input.c_str(), error);
      return 1;
    }
  }
  hexir_status_t st =
      hexir_program_emit_file(program, placement.c_str(), flags, out.c_str());
  if (st != HEXIR_OK) {
    std::fprintf(stderr, "%s\n", hexir_program_last_error(program));
    hexir_program_release(program);
    return 1;
  }
  hexir_program_release(program);
  return 0;
}
