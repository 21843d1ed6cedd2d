// Failure convention of the harness (results/naive_cycle4/include/playground/utils.hpp:6-14): print
// the failed condition with file and line to stderr and exit.  Used only by the driver and the
// version files; the library underneath returns status codes.
#pragma once

#include <cstdio>
#include <cstdlib>

#define PLAYGROUND_CHECK(condition)                                                                 \
    do {                                                                                            \
        if (!(condition)) {                                                                         \
            std::fprintf(stderr, "[Playground] Check failed at %s:%d for \"%s\"\n", __FILE__, __LINE__, \
                         #condition);                                                               \
            std::exit(EXIT_FAILURE);                                                                \
        }                                                                                           \
    } while (0)
