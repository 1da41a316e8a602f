// Minimal stderr logger standing in for QuasarML's spdlog logger
// (QuasarML/src/Common/Logger.h); level from the QSML_LOG environment
// variable (trace, debug, info, warn, error; default warn).
#pragma once

#include "Types.h"

namespace QuasarML {

class QS_API Logger {
public:
    enum Level { Trace = 0, Debug, Info, Warn, Error, Off };
    static void init();
    static void shutdown();
    static void log(Level level, const char* fmt, ...);
    static Level level();
};

}  // namespace QuasarML

#define LOG_TRACE(...) ::QuasarML::Logger::log(::QuasarML::Logger::Trace, __VA_ARGS__)
#define LOG_DEBUG(...) ::QuasarML::Logger::log(::QuasarML::Logger::Debug, __VA_ARGS__)
#define LOG_INFO(...) ::QuasarML::Logger::log(::QuasarML::Logger::Info, __VA_ARGS__)
#define LOG_WARN(...) ::QuasarML::Logger::log(::QuasarML::Logger::Warn, __VA_ARGS__)
#define LOG_ERROR(...) ::QuasarML::Logger::log(::QuasarML::Logger::Error, __VA_ARGS__)
