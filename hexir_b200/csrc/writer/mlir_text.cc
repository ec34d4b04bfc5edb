// mlir_text.cc -- parser for the textual program subset the reference's
// runtime tests are written in (runtime/test/*.mlir, bench/gemm/*.mlir):
//
//   func.func @main() {
//     %a = hexir.constant dense<[[3.0, 1.0], [2.0, 2.0]]> : tensor<2x2xf64>
//     %b = hexir.constant dense<2.000000e+00> : tensor<128x128xf64>
//     %m = hexir.linear %a, %b : tensor<2x2xf64>
//     %n = hexir.linear %x, %w : (tensor<8x16xf64>, tensor<16x4xf64>) -> tensor<8x4xf64>
//     %s = hexir.add %m, %b : tensor<2x2xf64>
//     %r = hexir.relu %s : tensor<2x2xf64>
//     %g = hexir.gelu %r : tensor<2x2xf64>
//     hexir.print %r : tensor<2x2xf64>
//     return
//   }
//
// Binary ops accept `: T` or the functional form `(T1, T2) -> T3`, as the
// reference parser does (compiler/Dialect/Hexir/IR/HexirDialect.cpp:238-264).
// The unary activations the dialect declares (leaky_relu, elu, sigmoid, tanh,
// softmax, gelu, swish, mish; printed like relu, HexirDialect.cpp:377-390)
// parse into the program; the writer serializes them only on request, else
// it refuses them as the reference serializer does.  Any other hexir op is
// refused here with that serializer's message "cannot serialize this op into
// a host program" (ModuleSerializer.cpp:368).

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "hexir_b200/hxb_writer.h"

namespace {

bool is_activation(const std::string &op) {
  static const char *const names[] = {
      "hexir.leaky_relu", "hexir.elu",     "hexir.sigmoid", "hexir.tanh",
      "hexir.softmax",    "hexir.gelu",    "hexir.swish",   "hexir.mish"};
  for (const char *n : names)
    if (op == n)
      return true;
  return false;
}

struct Parser {
  const char *s;
  size_t pos = 0, line = 1;
  std::string error;
  hexir_program_t *prog = nullptr;
  std::map<std::string, int32_t> names;

  explicit Parser(const char *text) : s(text) {}

  bool fail(const std::string &msg) {
    if (error.empty())
      error = "line " + std::to_string(line) + ": " + msg;
    return false;
  }

  void skip() {
    for (;;) {
      while (s[pos] && std::isspace(static_cast<unsigned char>(s[pos]))) {
        if (s[pos] == '\n')
          ++line;
        ++pos;
      }
      if (s[pos] == '/' && s[pos + 1] == '/') {
        while (s[pos] && s[pos] != '\n')
          ++pos;
        continue;
      }
      return;
    }
  }

  bool peek(const char *tok) {
    skip();
    return std::strncmp(s + pos, tok, std::strlen(tok)) == 0;
  }

  bool eat(const char *tok) {
    if (!peek(tok))
      return false;
    pos += std::strlen(tok);
    return true;
  }

  bool expect(const char *tok) {
    if (eat(tok))
      return true;
    return fail(std::string("expected '") + tok + "'");
  }

  std::string ident() {
    skip();
    size_t b = pos;
    while (s[pos] && (std::isalnum(static_cast<unsigned char>(s[pos])) ||
                      s[pos] == '_' || s[pos] == '.' || s[pos] == '$'))
      ++pos;
    return std::string(s + b, pos - b);
  }

  bool value_name(std::string *out) {
    skip();
    if (s[pos] != '%')
      return fail("expected an SSA value");
    ++pos;
    *out = ident();
    if (out->empty())
      return fail("expected an SSA value name");
    return true;
  }

  bool operand(int32_t *out) {
    std::string name;
    if (!value_name(&name))
      return false;
    auto it = names.find(name);
    if (it == names.end())
      return fail("use of undefined value %" + name);
    *out = it->second;
    return true;
  }

  // tensor<RxCxf64>
  bool tensor_type(uint32_t *rows, uint32_t *cols) {
    if (!expect("tensor") || !expect("<"))
      return false;
    skip();
    size_t b = pos;
    while (s[pos] && s[pos] != '>')
      ++pos;
    if (!s[pos])
      return fail("unterminated tensor type");
    std::string body(s + b, pos - b);
    ++pos;
    std::vector<std::string> parts;
    size_t start = 0;
    for (size_t i = 0; i <= body.size(); ++i)
      if (i == body.size() || body[i] == 'x') {
        parts.push_back(body.substr(start, i - start));
        start = i + 1;
      }
    if (parts.size() != 3 || parts[2] != "f64")
      return fail("only rank-2 f64 tensors are supported (got tensor<" + body +
                  ">)");
    for (int i = 0; i < 2; ++i)
      for (char c : parts[i])
        if (!std::isdigit(static_cast<unsigned char>(c)))
          return fail("bad tensor dimension '" + parts[i] + "'");
    *rows = static_cast<uint32_t>(std::strtoul(parts[0].c_str(), nullptr, 10));
    *cols = static_cast<uint32_t>(std::strtoul(parts[1].c_str(), nullptr, 10));
    return true;
  }

  // `: T` or `: (T1, T2) -> T3`; returns the result type.
  bool op_type(int operands, uint32_t *rows, uint32_t *cols) {
    if (!expect(":"))
      return false;
    if (eat("(")) {
      uint32_t r, c;
      for (int i = 0; i < operands; ++i) {
        if (i && !expect(","))
          return false;
        if (!tensor_type(&r, &c))
          return false;
      }
      if (!expect(")") || !expect("->"))
        return false;
    }
    return tensor_type(rows, cols);
  }

  bool number(double *out) {
    skip();
    char *end = nullptr;
    *out = std::strtod(s + pos, &end);
    if (end == s + pos)
      return fail("expected a number");
    pos = static_cast<size_t>(end - s);
    return true;
  }

  bool literal(std::vector<double> *flat, int *depth_seen, int depth) {
    if (eat("[")) {
      if (depth + 1 > *depth_seen)
        *depth_seen = depth + 1;
      if (eat("]"))
        return true;
      do {
        if (!literal(flat, depth_seen, depth + 1))
          return false;
      } while (eat(","));
      return expect("]");
    }
    if (eat("true") || eat("false"))
      return fail("boolean literals are not f64");
    double v;
    if (!number(&v))
      return false;
    flat->push_back(v);
    return true;
  }

  bool statement() {
    if (eat("return")) {
      // `return` or `return %x : T` -- a result is not part of the program.
      skip();
      if (s[pos] == '%') {
        std::string ignored;
        value_name(&ignored);
        uint32_t r, c;
        if (eat(":") && !tensor_type(&r, &c))
          return false;
      }
      return true;
    }
    if (eat("hexir.print")) {
      int32_t v;
      uint32_t r, c;
      if (!operand(&v) || !expect(":") || !tensor_type(&r, &c))
        return false;
      if (hexir_program_print(prog, v) != HEXIR_OK)
        return fail(hexir_program_last_error(prog));
      return true;
    }
    std::string result;
    if (!value_name(&result) || !expect("="))
      return false;
    std::string op = ident();
    int32_t id = -1;
    uint32_t rows = 0, cols = 0;
    if (op == "hexir.constant") {
      if (!expect("dense") || !expect("<"))
        return false;
      std::vector<double> flat;
      int depth = 0;
      if (!literal(&flat, &depth, 0) || !expect(">") || !expect(":") ||
          !tensor_type(&rows, &cols))
        return false;
      const size_t count = static_cast<size_t>(rows) * cols;
      if (depth == 0 && flat.size() == 1)
        id = hexir_program_splat(prog, flat[0], rows, cols);
      else if (flat.size() == count)
        id = hexir_program_constant(prog, flat.data(), rows, cols);
      else
        return fail("dense literal has " + std::to_string(flat.size()) +
                    " elements, type needs " + std::to_string(count));
    } else if (op == "hexir.linear" || op == "hexir.add") {
      int32_t a, b;
      if (!operand(&a) || !expect(",") || !operand(&b) ||
          !op_type(2, &rows, &cols))
        return false;
      id = op == "hexir.linear" ? hexir_program_linear(prog, a, b)
                                : hexir_program_add(prog, a, b);
    } else if (op == "hexir.relu") {
      int32_t a;
      if (!operand(&a) || !op_type(1, &rows, &cols))
        return false;
      id = hexir_program_relu(prog, a);
    } else if (is_activation(op)) {
      int32_t a;
      if (!operand(&a) || !op_type(1, &rows, &cols))
        return false;
      id = hexir_program_activation(prog, op.c_str(), a);
    } else if (op.rfind("hexir.", 0) == 0) {
      return fail("'" + op + "': cannot serialize this op into a host program");
    } else {
      return fail("unsupported operation '" + op + "'");
    }
    if (id < 0)
      return fail(hexir_program_last_error(prog));
    names[result] = id;
    return true;
  }

  bool function() {
    if (!expect("func.func"))
      return false;
    skip();
    if (s[pos] != '@')
      return fail("expected @name");
    ++pos;
    std::string name = ident();
    if (name.empty())
      return fail("expected a function name");
    if (!expect("(") || !expect(")"))
      return fail("functions take no arguments in a host program");
    if (!expect("{"))
      return false;
    if (hexir_program_begin_function(prog, name.c_str()) != HEXIR_OK)
      return fail("bad function name");
    names.clear();
    while (!eat("}")) {
      skip();
      if (!s[pos])
        return fail("unterminated function body");
      if (!statement())
        return false;
    }
    return true;
  }

  bool module() {
    bool wrapped = eat("module");
    if (wrapped && !expect("{"))
      return false;
    for (;;) {
      skip();
      if (wrapped && eat("}"))
        return true;
      if (!s[pos])
        return wrapped ? fail("unterminated module") : true;
      if (!function())
        return false;
    }
  }
};

}  // namespace

extern "C" hexir_status_t hexir_program_parse(const char *text,
                                              hexir_program_t **out,
                                              char *error, size_t error_size) {
  if (!text || !out)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out = nullptr;
  Parser p(text);
  p.prog = hexir_program_create();
  if (!p.prog)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  if (!p.module()) {
    if (error && error_size)
      std::snprintf(error, error_size, "%s", p.error.c_str());
    hexir_program_release(p.prog);
    return HEXIR_ERROR_INVALID_ARGUMENT;
  }
  *out = p.prog;
  return HEXIR_OK;
}
