// eg_host.h -- internal host helpers shared by eg_host.cpp and eg_runtime.cu.
#pragma once
#include <stdint.h>

#include "emberglass.h"

namespace eg {
uint64_t stream_at(uint64_t seed, uint64_t k);
void fill_normal(float* out, int64_t n, uint64_t seed, double stdv, int64_t start);
void rope_tables(int max_ctx, int hd, double theta, float* cosT, float* sinT);
// Records the message for eg_last_error() and returns the status.
eg_status fail(eg_status st, const char* fmt, ...);
}  // namespace eg
