/*
 * status.h -- result codes of every hexir runtime entry point.
 *
 * Same eight codes, same numeric values and same strings as the reference
 * runtime (runtime/include/hexir_runtime/status.h:9-18,
 * runtime/src/status.c:3-15): callers that compare against these values, and
 * tests that grep the strings, keep working unchanged.
 */
#ifndef HEXIR_RUNTIME_STATUS_H
#define HEXIR_RUNTIME_STATUS_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HEXIR_OK = 0,
  HEXIR_ERROR_INVALID_ARGUMENT = 1,
  HEXIR_ERROR_NOT_FOUND = 2,
  HEXIR_ERROR_OUT_OF_MEMORY = 3,
  HEXIR_ERROR_UNIMPLEMENTED = 4,
  HEXIR_ERROR_INVALID_MODULE = 5,
  HEXIR_ERROR_IO = 6,
  HEXIR_ERROR_DEVICE = 7,
} hexir_status_t;

/* "ok", "invalid argument", "not found", "out of memory", "unimplemented",
 * "invalid module", "io error", "device error"; "unknown" otherwise. */
const char *hexir_status_string(hexir_status_t status);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_STATUS_H */
