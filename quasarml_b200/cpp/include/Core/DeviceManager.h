// Process-wide registry of CUDA devices (QuasarML/src/Core/DeviceManager.h).
#pragma once

#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "Device.h"

namespace QuasarML {

class QS_API DeviceManager {
public:
    static DeviceManager& instance();
    u32 device_count() const { return _device_count; }
    Device* get(u32 device_id = 0);  // nullptr if the device does not exist or fails to open
    std::vector<std::string> device_names() const;
    void set_default(u32 device_id);
    u32 get_default() const { return _default_device; }
    void shutdown();
    ~DeviceManager();

private:
    DeviceManager();
    DeviceManager(const DeviceManager&) = delete;
    DeviceManager& operator=(const DeviceManager&) = delete;
    mutable std::mutex _mutex;
    std::unordered_map<u32, std::unique_ptr<Device>> _devices;
    u32 _device_count = 0;
    u32 _default_device = 0;
    bool _shutdown = false;
};

}  // namespace QuasarML
