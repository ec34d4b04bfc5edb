/*
 * module.h -- the .hxb container: header, section table, 8-byte aligned
 * payloads, all little-endian, offsets absolute from the start of the file.
 *
 * The byte layout is the reference's version 3 format
 * (runtime/include/hexir_runtime/module.h:28-57) so that modules move freely
 * between the two runtimes; the loader API (module.h:63-77) is the same.
 *
 * extension: section kind 5, HEXIR_SECTION_LAUNCH, describes how each
 * executable is launched by this library (fusion, device ordinal, row
 * sharding).  The reference loader looks sections up by kind and skips kinds
 * it does not know (runtime/src/module/module.c:124-139), so a module with a
 * LAUNCH section is still a valid version 3 module.
 */
#ifndef HEXIR_RUNTIME_MODULE_H
#define HEXIR_RUNTIME_MODULE_H

#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

#define HEXIR_MODULE_MAGIC "HEXIRMOD"
#define HEXIR_MODULE_MAGIC_SIZE 8
#define HEXIR_MODULE_VERSION 3u

typedef enum {
  HEXIR_SECTION_SYMBOLS = 1,     /* entry points: name -> program offset */
  HEXIR_SECTION_PROGRAM = 2,     /* flat command list */
  HEXIR_SECTION_RODATA = 3,      /* constants, used in place from the map */
  HEXIR_SECTION_EXECUTABLES = 4, /* kernel descriptors + device images */
  HEXIR_SECTION_LAUNCH = 5,      /* extension: per-executable launch info */
} hexir_section_kind_t;

typedef struct {
  char magic[HEXIR_MODULE_MAGIC_SIZE];
  uint32_t version;
  uint32_t flags;
  uint32_t section_count;
  uint32_t reserved;
} hexir_module_header_t; /* 24 bytes */

typedef struct {
  uint32_t kind;
  uint32_t flags;
  uint64_t offset; /* absolute file offset */
  uint64_t size;
} hexir_section_entry_t; /* 24 bytes */

typedef struct hexir_module_t hexir_module_t;

/* mmap a module read-only and validate the header and every section bound.
 * IO for an unreadable or empty file, INVALID_MODULE for a bad one. */
hexir_status_t hexir_module_load_file(const char *path, hexir_module_t **out);
void hexir_module_release(hexir_module_t *module);

uint32_t hexir_module_version(const hexir_module_t *module);
uint32_t hexir_module_section_count(const hexir_module_t *module);
const hexir_section_entry_t *hexir_module_section_at(const hexir_module_t *module,
                                                     uint32_t index);

/* First section of `kind`; `*data` points into the mapping (zero copy). */
hexir_status_t hexir_module_section(const hexir_module_t *module,
                                    hexir_section_kind_t kind,
                                    const void **data, uint64_t *size);

/* "symbols", "program", "rodata", "executables", "launch", else "unknown". */
const char *hexir_section_kind_string(uint32_t kind);

/* extension: load a module from memory (the bytes are copied). */
hexir_status_t hexir_module_load_memory(const void *data, uint64_t size,
                                        hexir_module_t **out);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_MODULE_H */
