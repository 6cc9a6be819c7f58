#pragma once
// Compile-time leveled logging to stderr.
// Mirrors the reference interface include/gfd/log.h:15-29 (same macro names and
// level meaning: 0 silent, 1 errors, 2 info (default), 3 debug).

#include <cstdio>

#ifndef GFD_LOG_LEVEL
#define GFD_LOG_LEVEL 2
#endif

#define GFD_LOG_ERROR(...)                                                    \
    do {                                                                      \
        if (GFD_LOG_LEVEL >= 1) { fputs("[GFD ERROR] ", stderr); fprintf(stderr, __VA_ARGS__); } \
    } while (0)

#define GFD_LOG_INFO(...)                                                     \
    do {                                                                      \
        if (GFD_LOG_LEVEL >= 2) { fputs("[GFD] ", stderr); fprintf(stderr, __VA_ARGS__); } \
    } while (0)

#define GFD_LOG_DEBUG(...)                                                    \
    do {                                                                      \
        if (GFD_LOG_LEVEL >= 3) { fputs("[GFD DBG] ", stderr); fprintf(stderr, __VA_ARGS__); } \
    } while (0)
