// module.cc -- .hxb loading (include/hexir_runtime/module.h).
//
// Same contract as the reference loader (runtime/src/module/module.c:36-139):
// the file is mapped read-only, the header (magic, version 3) and every
// section's bounds are validated before any pointer is handed out, sections
// are found by kind, and unknown kinds are ignored.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "hexir_runtime/module.h"

#include "module_internal.h"

struct hexir_module_t {
  void *mapping = nullptr;  // mmap'd file, or nullptr for a memory copy
  uint8_t *copy = nullptr;  // owned bytes for hexir_module_load_memory
  const uint8_t *base = nullptr;
  size_t size = 0;
  hexir_module_header_t header;  // copied: the mapping may be unaligned-safe
  const hexir_section_entry_t *sections = nullptr;
  // Runtime state tied to the module's lifetime (pinned RODATA); released
  // before the bytes are unmapped.
  std::mutex attach_mu;
  void *attached = nullptr;
  void (*detach)(void *) = nullptr;
};

namespace hexir {

void *module_attached(const hexir_module_t *module, void *(*make)(const hexir_module_t *),
                      void (*detach)(void *)) {
  auto *m = const_cast<hexir_module_t *>(module);
  std::lock_guard<std::mutex> lock(m->attach_mu);
  if (!m->attached) {
    m->attached = make(module);
    if (m->attached)
      m->detach = detach;
  }
  return m->attached;
}

}  // namespace hexir

namespace {

hexir_status_t validate(hexir_module_t *m) {
  if (m->size < sizeof(hexir_module_header_t))
    return HEXIR_ERROR_INVALID_MODULE;
  std::memcpy(&m->header, m->base, sizeof(m->header));
  if (std::memcmp(m->header.magic, HEXIR_MODULE_MAGIC,
                  HEXIR_MODULE_MAGIC_SIZE) != 0)
    return HEXIR_ERROR_INVALID_MODULE;
  if (m->header.version != HEXIR_MODULE_VERSION)
    return HEXIR_ERROR_INVALID_MODULE;
  const uint64_t table =
      static_cast<uint64_t>(m->header.section_count) *
      sizeof(hexir_section_entry_t);
  if (sizeof(hexir_module_header_t) + table > m->size)
    return HEXIR_ERROR_INVALID_MODULE;
  m->sections = reinterpret_cast<const hexir_section_entry_t *>(
      m->base + sizeof(hexir_module_header_t));
  // Offsets come off disk: bound every payload before trusting it.  The
  // format puts every section on an 8-byte boundary (the serializer pads)
  // and the tables are read in place, so an unaligned section is refused.
  for (uint32_t i = 0; i < m->header.section_count; ++i) {
    const hexir_section_entry_t &s = m->sections[i];
    if (s.offset > m->size || s.size > m->size - s.offset || s.offset % 8 != 0)
      return HEXIR_ERROR_INVALID_MODULE;
  }
  return HEXIR_OK;
}

}  // namespace

extern "C" {

const char *hexir_section_kind_string(uint32_t kind) {
  switch (kind) {
  case HEXIR_SECTION_SYMBOLS: return "symbols";
  case HEXIR_SECTION_PROGRAM: return "program";
  case HEXIR_SECTION_RODATA: return "rodata";
  case HEXIR_SECTION_EXECUTABLES: return "executables";
  case HEXIR_SECTION_LAUNCH: return "launch";
  }
  return "unknown";
}

hexir_status_t hexir_module_load_file(const char *path, hexir_module_t **out) {
  if (!path || !out)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out = nullptr;
  int fd = open(path, O_RDONLY);
  if (fd < 0)
    return HEXIR_ERROR_IO;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return HEXIR_ERROR_IO;
  }
  void *base = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ,
                    MAP_PRIVATE, fd, 0);
  close(fd);
  if (base == MAP_FAILED)
    return HEXIR_ERROR_IO;
  auto *m = new (std::nothrow) hexir_module_t;
  if (!m) {
    munmap(base, static_cast<size_t>(st.st_size));
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  m->mapping = base;
  m->base = static_cast<const uint8_t *>(base);
  m->size = static_cast<size_t>(st.st_size);
  hexir_status_t status = validate(m);
  if (status != HEXIR_OK) {
    hexir_module_release(m);
    return status;
  }
  *out = m;
  return HEXIR_OK;
}

hexir_status_t hexir_module_load_memory(const void *data, uint64_t size,
                                        hexir_module_t **out) {
  if (!data || !out)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out = nullptr;
  if (size == 0)
    return HEXIR_ERROR_IO;
  auto *m = new (std::nothrow) hexir_module_t;
  if (!m)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  // 64-byte aligned copy so section payloads keep their 8-byte alignment.
  m->copy = static_cast<uint8_t *>(std::aligned_alloc(64, (size + 63) & ~63ull));
  if (!m->copy) {
    delete m;
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  std::memcpy(m->copy, data, size);
  m->base = m->copy;
  m->size = size;
  hexir_status_t status = validate(m);
  if (status != HEXIR_OK) {
    hexir_module_release(m);
    return status;
  }
  *out = m;
  return HEXIR_OK;
}

void hexir_module_release(hexir_module_t *module) {
  if (!module)
    return;
  if (module->attached && module->detach)
    module->detach(module->attached);
  if (module->mapping)
    munmap(module->mapping, module->size);
  std::free(module->copy);
  delete module;
}

uint32_t hexir_module_version(const hexir_module_t *m) {
  return m ? m->header.version : 0u;
}

uint32_t hexir_module_section_count(const hexir_module_t *m) {
  return m ? m->header.section_count : 0u;
}

const hexir_section_entry_t *hexir_module_section_at(const hexir_module_t *m,
                                                     uint32_t index) {
  if (!m || index >= m->header.section_count)
    return nullptr;
  return &m->sections[index];
}

hexir_status_t hexir_module_section(const hexir_module_t *m,
                                    hexir_section_kind_t kind,
                                    const void **data, uint64_t *size) {
  if (!m || !data || !size)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  for (uint32_t i = 0; i < m->header.section_count; ++i) {
    if (m->sections[i].kind == static_cast<uint32_t>(kind)) {
      *data = m->base + m->sections[i].offset;
      *size = m->sections[i].size;
      return HEXIR_OK;
    }
  }
  *data = nullptr;
  *size = 0;
  return HEXIR_ERROR_NOT_FOUND;
}

}  // extern "C"
