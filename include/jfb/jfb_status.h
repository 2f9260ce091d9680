/*
 * Status record shared by every jfb_* entry point. It mirrors the loader's
 * jf_status (runtime/engines/native/include/jetsonfabric/engine.h:50-62): a
 * code plus a NUL-terminated message, returned by value, never an exception
 * across the ABI.
 */
#ifndef JFB_STATUS_H
#define JFB_STATUS_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum jfb_status_code {
    JFB_STATUS_OK = 0,
    /* Invalid input: the reference engine throws std::invalid_argument for
     * these and the stage executor maps them to HTTP 400
     * (runtime/adapters/native_stage_executor.cpp:129-134). */
    JFB_STATUS_INVALID_ARGUMENT = 1,
    JFB_STATUS_IO_ERROR = 2,
    JFB_STATUS_FORMAT_ERROR = 3,
    JFB_STATUS_NOT_FOUND = 4,
    JFB_STATUS_OUT_OF_MEMORY = 5,
    /* Any other execution failure (HTTP 502 in the reference executor). */
    JFB_STATUS_EXECUTION_FAILED = 6,
    JFB_STATUS_CUDA_ERROR = 7,
    JFB_STATUS_UNSUPPORTED = 8,
    /* A bounded device-side or peer wait gave up. */
    JFB_STATUS_TIMEOUT = 9
} jfb_status_code;

typedef struct jfb_status {
    jfb_status_code code;
    char message[256];
} jfb_status;

const char * jfb_status_code_name(jfb_status_code code);

#ifdef __cplusplus
}
#endif

#endif
