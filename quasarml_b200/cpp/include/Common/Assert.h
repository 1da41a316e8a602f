// Error convention of QuasarML (QuasarML/src/Common/Assert.h:8-20): failed
// checks throw std::runtime_error.
#pragma once

#include <stdexcept>
#include <string>

namespace QuasarML {

#define QS_ASSERT(condition, message)                                                          \
    do {                                                                                       \
        if (!(condition)) throw std::runtime_error(std::string("Assertion failed: ") + (message)); \
    } while (0)

#define QS_CHECK(condition)                                                    \
    do {                                                                       \
        if (!(condition)) throw std::runtime_error("Check failed: " #condition); \
    } while (0)

}  // namespace QuasarML
