// Logging and status helpers shared by the host code of librfdetr.
#pragma once

#include "rfdetr.h"

#include <cuda_runtime.h>

// printf-style log through the process-global callback installed with
// rfdetr_set_log_callback (reference semantics: src/common.cpp:33-60).
void rfdetr_logf(rfdetr_log_level lvl, const char* fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;

// Logs a CUDA error with context; returns true if `e` is an error.
bool rfdetr_cuda_failed(cudaError_t e, const char* what, const char* file, int line);

#define RFB_CUDA_FAIL(expr) rfdetr_cuda_failed((expr), #expr, __FILE__, __LINE__)
