// A CUDA device as QuasarML sees it (QuasarML/src/Core/Device.h): owns a
// qsml_ctx (stream + caching allocator) of libqsml_cuda.so in place of the
// Vulkan backend.  GLSL kernel creation (create_kernel / get_kernel) has no
// counterpart: every op is a precompiled sm_100a kernel.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "../Common/Types.h"

struct qsml_ctx;

namespace QuasarML {

class Tensor;

class QS_API Device {
public:
    Device(const std::string& name, u32 device_index = 0);
    ~Device();
    Device(const Device&) = delete;
    Device& operator=(const Device&) = delete;

    bool is_valid() const { return _ctx != nullptr; }
    u32 device_index() const { return _device_index; }
    const std::string& name() const { return _name; }
    qsml_ctx* ctx() const { return _ctx; }

    std::shared_ptr<Tensor> create_tensor(const std::vector<u32>& shape, DataType dtype = DataType::F32,
                                          bool host_visible = false);

    // Elementwise fusion: while on (set_fusion(true), or between begin_batch
    // and end_batch) elementwise ops on F32/F16 tensors return deferred
    // results that evaluate as one fused kernel on first access.
    void set_fusion(bool on);
    bool fusion() const { return _fusion; }
    // Overlap of independent reductions, layer norms, softmaxes, gathers and
    // elementwise ops on the device's stream (a call sharing no buffer with
    // the kernels still running before it starts at once; qsml_set_overlap).
    // On by default (the stream is the library's own; QSML_OVERLAP=0 at
    // start-up, or set_overlap(false), turns it off).
    void set_overlap(bool on);
    bool defer_elementwise() const { return _fusion || _in_batch; }

    // Work is enqueued in order on one stream; a batch additionally defers
    // and fuses elementwise ops (see set_fusion).
    void begin_batch();
    void end_batch();
    void flush_pending();
    void synchronize();
    void wait_idle();

    // Throws std::runtime_error with the library's message if st != 0.
    void check(int st) const;
    // Tensors hold this to learn whether the device still exists.
    std::weak_ptr<int> alive_token() const { return _alive; }

private:
    qsml_ctx* _ctx = nullptr;
    std::shared_ptr<int> _alive;
    std::string _name;
    u32 _device_index = 0;
    bool _in_batch = false;
    bool _fusion = false;
};

}  // namespace QuasarML
