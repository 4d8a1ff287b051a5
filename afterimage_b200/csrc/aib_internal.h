// Internal helpers shared by the library's translation units.
#pragma once
#include <cstdint>

#include "afterimage_b200.h"

#define AIB_API extern "C" __attribute__((visibility("default")))

// Records msg as this thread's last error (read back by aib_last_error()).
void aib_set_error(const char *msg);
void aib_set_errorf(const char *fmt, ...);
