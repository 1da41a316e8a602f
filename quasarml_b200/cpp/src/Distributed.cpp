// Ops::all_reduce over qsml_group_init_all / qsml_allreduce.
#include <map>
#include <mutex>

#include "Common/Assert.h"
#include "Core/Device.h"
#include "Core/Tensor.h"
#include "Ops/Distributed.h"

namespace QuasarML {
namespace Ops {

namespace {

std::mutex g_mu;
std::map<std::vector<Device*>, qsml_group*> g_groups;  // device set -> group

qsml_group* group_for(const std::vector<Device*>& devs) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_groups.find(devs);
    if (it != g_groups.end()) return it->second;
    std::vector<qsml_ctx*> ctxs;
    for (Device* d : devs) ctxs.push_back(d->ctx());
    qsml_group* g = nullptr;
    const int st = qsml_group_init_all(ctxs.data(), static_cast<int32_t>(ctxs.size()), &g);
    if (st != QSML_OK) throw std::runtime_error(qsml_last_error(nullptr));
    g_groups[devs] = g;
    return g;
}

}  // namespace

void all_reduce(const std::vector<std::shared_ptr<Tensor>>& tensors, ReduceOp op) {
    QS_ASSERT(!tensors.empty(), "all_reduce needs at least one tensor");
    std::vector<Device*> devs;
    for (const auto& t : tensors) {
        QS_ASSERT(t && t->is_contiguous(), "all_reduce needs contiguous tensors");
        QS_ASSERT(t->shape() == tensors[0]->shape() && t->dtype() == tensors[0]->dtype(),
                  "all_reduce needs equal shapes and dtypes");
        for (Device* d : devs) QS_ASSERT(d != t->device(), "all_reduce needs one tensor per device");
        devs.push_back(t->device());
    }
    qsml_group* g = group_for(devs);
    // Each device's queued work (including deferred results) comes first.
    for (const auto& t : tensors) t->materialize();
    const int32_t n = static_cast<int32_t>(tensors.size());
    if (n > 1) QS_ASSERT(qsml_group_start() == QSML_OK, "qsml_group_start failed");
    int first_err = QSML_OK;
    Device* err_dev = nullptr;
    for (int32_t i = 0; i < n; ++i) {
        const int st = qsml_allreduce(g, i, tensors[i]->data(), static_cast<int64_t>(tensors[i]->numel()),
                                      static_cast<int32_t>(tensors[i]->dtype()), static_cast<int32_t>(op));
        if (st != QSML_OK && first_err == QSML_OK) {
            first_err = st;
            err_dev = devs[i];
        }
    }
    if (n > 1) {
        const int st = qsml_group_end();
        if (st != QSML_OK && first_err == QSML_OK) throw std::runtime_error(qsml_last_error(nullptr));
    }
    if (first_err != QSML_OK) err_dev->check(first_err);
}

void release_device_groups() {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& kv : g_groups) qsml_group_destroy(kv.second);
    g_groups.clear();
}

}  // namespace Ops
}  // namespace QuasarML
