/* Stub XRT types for compiling the reference's libonpu host code (onpu_api.cpp, onpu_cpu.cpp)
 * WITHOUT an NPU. Test infrastructure only: every device-touching call is inert, and the
 * reference's Device::init() never reaches them because no gemv.xclbin exists on this machine,
 * so onpu_ok() returns 0. Only the host-only exports (onpu_geometry2, onpu_pack,
 * onpu_quant_dequant, onpu_moe_act, onpu_moe_sum) are used from the resulting library. */
#pragma once
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <string>

enum ert_cmd_state { ERT_CMD_STATE_NEW = 1, ERT_CMD_STATE_COMPLETED = 4, ERT_CMD_STATE_ERROR = 5 };
enum xclBOSyncDirection { XCL_BO_SYNC_BO_TO_DEVICE = 0, XCL_BO_SYNC_BO_FROM_DEVICE = 1 };

namespace xrt {
struct uuid {};
struct xclbin {
    xclbin() = default;
    explicit xclbin(const std::string &) {}
    uuid get_uuid() const { return {}; }
};
struct device {
    device() = default;
    explicit device(unsigned) {}
    void register_xclbin(const xclbin &) {}
};
struct hw_context {
    hw_context() = default;
    hw_context(const device &, const uuid &) {}
};
struct kernel {
    kernel() = default;
    kernel(const hw_context &, const std::string &) {}
    int group_id(int) const { return 0; }
};
struct bo {
    enum class flags : uint32_t { normal = 0, cacheable = 1, host_only = 2 };
    bo() = default;
    bo(const device &, size_t, flags, int) {}
    template <typename T> T map() { return nullptr; }
    void sync(xclBOSyncDirection) {}
    void write(const void *) {}
};
struct run {
    run() = default;
    explicit run(const kernel &) {}
    template <typename T> void set_arg(int, const T &) {}
    void start() {}
    ert_cmd_state wait(std::chrono::milliseconds) { return ERT_CMD_STATE_ERROR; }
};
}  // namespace xrt
