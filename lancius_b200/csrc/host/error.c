/* Thread-local error code (reference: bleeding/v11A1/src/core/lancius_error.c:5-34). */
#include "lancius/lancius_error.h"

static _Thread_local lancius_error tl_err = LANCIUS_ERROR_OK;

void lancius_set_error(lancius_error err) { tl_err = err; }
lancius_error lancius_get_error(void) { return tl_err; }
void lancius_clear_error(void) { tl_err = LANCIUS_ERROR_OK; }

const char* lancius_error_string(lancius_error err) {
    static const char* names[] = { "success", "out of memory", "null pointer", "shape mismatch",
        "unsupported op", "unsupported dtype", "invalid model", "version mismatch", "io error",
        "overflow", "internal error" };
    int i = -(int)err;
    return (i >= 0 && i <= 10) ? names[i] : "unknown error";
}
