// Ops::all_reduce over qsml_group_init_all / qsml_allreduce.
#include <cmath>
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

namespace {

std::vector<std::shared_ptr<Tensor>> sharded_impl(const std::vector<std::shared_ptr<Tensor>>& blocks, ReduceOp op,
                                                  int32_t axis, bool keepdims) {
    QS_ASSERT(!blocks.empty(), "sharded_reduce needs at least one block");
    QS_ASSERT(op == ReduceOp::Sum || op == ReduceOp::Mean || op == ReduceOp::Max || op == ReduceOp::Min,
              "sharded_reduce supports sum, mean, max and min");
    const auto& b0 = blocks[0];
    QS_ASSERT(b0 && b0->rank() >= 1, "sharded_reduce needs blocks with a row axis");
    std::vector<Device*> devs;
    u64 global_rows = 0, row_elems = 1;
    for (size_t d = 1; d < b0->rank(); ++d) row_elems *= b0->dim(d);
    for (const auto& b : blocks) {
        QS_ASSERT(b && b->dtype() == b0->dtype() && b->rank() == b0->rank(), "blocks must agree in dtype and rank");
        for (size_t d = 1; d < b->rank(); ++d) QS_ASSERT(b->dim(d) == b0->dim(d), "blocks must agree beyond the row axis");
        for (Device* d : devs) QS_ASSERT(d != b->device(), "sharded_reduce needs one block per device");
        devs.push_back(b->device());
        global_rows += b->dim(0);
    }
    const int32_t code = static_cast<int32_t>(op);
    auto reduced = [&](const std::shared_ptr<Tensor>& b) {
        std::vector<u32> s;
        if (axis == QSML_AXIS_ALL) return std::vector<u32>{1};
        for (size_t d = 0; d < b->rank(); ++d) {
            if (static_cast<int32_t>(d) != axis) s.push_back(b->dim(d));
            else if (keepdims) s.push_back(1);
        }
        if (s.empty()) s.push_back(1);
        return s;
    };
    std::vector<std::shared_ptr<Tensor>> outs;
    if (axis != QSML_AXIS_ALL && axis != 0) {
        // each device's rows of the result: no exchange
        for (size_t i = 0; i < blocks.size(); ++i) {
            auto out = devs[i]->create_tensor(reduced(blocks[i]), b0->dtype());
            blocks[i]->materialize();
            qsml_tdesc dx = blocks[i]->desc(), dout = out->desc();
            devs[i]->check(qsml_reduce(devs[i]->ctx(), code, &dx, axis, keepdims ? 1 : 0, &dout));
            outs.push_back(out);
        }
        return outs;
    }
    qsml_group* g = group_for(devs);
    std::vector<std::shared_ptr<Tensor>> parts;
    const auto oshape = reduced(b0);
    for (size_t i = 0; i < blocks.size(); ++i) {
        auto part = devs[i]->create_tensor(oshape, DataType::F32);
        qsml_tdesc dp = part->desc();
        if (blocks[i]->dim(0) == 0 && (op == ReduceOp::Max || op == ReduceOp::Min)) {
            const float v = op == ReduceOp::Max ? -INFINITY : INFINITY;  // no rows: the identity
            devs[i]->check(qsml_fill(devs[i]->ctx(), dp.data, &v, 4, static_cast<int64_t>(part->numel())));
        } else {
            blocks[i]->materialize();
            qsml_tdesc dx = blocks[i]->desc();
            devs[i]->check(qsml_reduce(devs[i]->ctx(), op == ReduceOp::Mean ? QSML_RED_SUM : code, &dx, axis,
                                       keepdims ? 1 : 0, &dp));
        }
        parts.push_back(part);
    }
    const bool bracket = blocks.size() > 1;
    if (bracket) QS_ASSERT(qsml_group_start() == QSML_OK, "qsml_group_start failed");
    int first_err = QSML_OK;
    size_t err_at = 0;
    for (size_t i = 0; i < parts.size(); ++i) {
        const int st = qsml_allreduce_partials(g, static_cast<int32_t>(i), code, parts[i]->data(),
                                               static_cast<int64_t>(parts[i]->numel()));
        if (st != QSML_OK && first_err == QSML_OK) {
            first_err = st;
            err_at = i;
        }
    }
    if (bracket && qsml_group_end() != QSML_OK && first_err == QSML_OK)
        throw std::runtime_error(qsml_last_error(nullptr));
    if (first_err != QSML_OK) devs[err_at]->check(first_err);
    const int64_t n = static_cast<int64_t>(axis == 0 ? global_rows : global_rows * row_elems);
    for (size_t i = 0; i < parts.size(); ++i) {
        auto out = devs[i]->create_tensor(oshape, b0->dtype());
        qsml_tdesc dp = parts[i]->desc(), dout = out->desc();
        devs[i]->check(qsml_finish_partial(devs[i]->ctx(), code, &dp, n, &dout));
        outs.push_back(out);
    }
    return outs;
}

}  // namespace

std::vector<std::shared_ptr<Tensor>> sharded_reduce(const std::vector<std::shared_ptr<Tensor>>& blocks, ReduceOp op,
                                                    i32 axis, bool keepdims) {
    QS_ASSERT(!blocks.empty() && blocks[0], "sharded_reduce needs at least one block");
    const i32 r = static_cast<i32>(blocks[0]->rank());
    if (axis < 0) axis += r;
    QS_ASSERT(axis >= 0 && axis < r, "Axis out of range");
    return sharded_impl(blocks, op, axis, keepdims);
}

std::vector<std::shared_ptr<Tensor>> sharded_reduce(const std::vector<std::shared_ptr<Tensor>>& blocks, ReduceOp op) {
    return sharded_impl(blocks, op, QSML_AXIS_ALL, false);
}

std::vector<std::shared_ptr<Tensor>> scatter_rows(const void* host, const std::vector<u32>& shape, DataType dtype,
                                                  const std::vector<Device*>& devices) {
    QS_ASSERT(!shape.empty() && !devices.empty(), "scatter_rows needs a row axis and a device");
    u64 row_bytes = dtype_size(dtype);
    for (size_t d = 1; d < shape.size(); ++d) row_bytes *= shape[d];
    std::vector<std::shared_ptr<Tensor>> blocks;
    for (size_t i = 0; i < devices.size(); ++i) {
        int64_t begin = 0, count = 0;
        QS_ASSERT(qsml_shard_rows(shape[0], static_cast<int32_t>(devices.size()), static_cast<int32_t>(i), &begin,
                                  &count) == QSML_OK, "qsml_shard_rows failed");
        std::vector<u32> s = shape;
        s[0] = static_cast<u32>(count);
        auto t = devices[i]->create_tensor(s, dtype);
        if (count > 0) t->upload(static_cast<const char*>(host) + begin * row_bytes, count * row_bytes);
        blocks.push_back(t);
    }
    return blocks;
}

void release_device_groups() {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& kv : g_groups) qsml_group_destroy(kv.second);
    g_groups.clear();
}

}  // namespace Ops
}  // namespace QuasarML
