// host_common.h -- helpers shared by the host model drivers.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/acb.h"

namespace acb {

void set_last_error(const std::string & e);

#define ACB_TRY(x)                 \
    do {                           \
        const acb_status s_ = (x); \
        if (s_ != ACB_OK) {        \
            return s_;             \
        }                          \
    } while (0)

// Value text of "key": in a flat JSON object (the lookup of qw3lm_json_int / _float / _bool,
// src/qwen3-lm.h:60-121), or nullptr.
inline const char * json_value(const char * j, const char * key) {
    char needle[128];
    snprintf(needle, sizeof(needle), "\"%s\"", key);
    const char * p = strstr(j, needle);
    if (!p) {
        return nullptr;
    }
    p = strchr(p + strlen(needle), ':');
    if (!p) {
        return nullptr;
    }
    p++;
    while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') {
        p++;
    }
    return p;
}

inline int json_int(const char * j, const char * key, int fb) {
    const char * v = json_value(j, key);
    return v ? atoi(v) : fb;
}

inline float json_float(const char * j, const char * key, float fb) {
    const char * v = json_value(j, key);
    return v ? (float) atof(v) : fb;
}

inline bool json_bool(const char * j, const char * key, bool fb) {
    const char * v = json_value(j, key);
    return v ? strncmp(v, "true", 4) == 0 : fb;
}

}  // namespace acb
