// Log macros (reference teco/ual/com/log.h:36-52).  Messages go to stderr when
// the environment variable TECOOPS_LOG_LEVEL is >= the message level
// (1 = errors, 2 = warnings, 3 = info); errors print by default.
#ifndef TECOOPS_B200_UAL_COM_LOG_H_
#define TECOOPS_B200_UAL_COM_LOG_H_

#include <cstdio>
#include <cstdlib>

namespace tecoops {
inline int logLevel() {
    static int lvl = [] {
        const char *e = std::getenv("TECOOPS_LOG_LEVEL");
        return e ? std::atoi(e) : 1;
    }();
    return lvl;
}
}  // namespace tecoops

#define TECO_LOG_AT(level, tag, ...)                                   \
    do {                                                               \
        if (::tecoops::logLevel() >= (level)) {                        \
            std::fprintf(stderr, "[tecoops %s] ", tag);                \
            std::fprintf(stderr, __VA_ARGS__);                         \
            std::fprintf(stderr, "\n");                                \
        }                                                              \
    } while (0)
#define TECO_ERROR(...) TECO_LOG_AT(1, "ERROR", __VA_ARGS__)
#define TECO_WARNING(...) TECO_LOG_AT(2, "WARNING", __VA_ARGS__)
#define TECO_LOG(...) TECO_LOG_AT(3, "INFO", __VA_ARGS__)

#endif  // TECOOPS_B200_UAL_COM_LOG_H_
