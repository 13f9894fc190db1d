// pydee.cpp -- the `pydee.Engine` binding, rebuilt over this library's C ABI.
//
// The reference exposes its engine to Python as a pybind11 module
// (dee.cpp/pydee/pydee.cpp); its DeepSeek-V4 layer calls
// Engine.moe_forward_batch_device / moe_forward_combined_device with raw
// device pointers (uintptr_t) and releases the GIL around the engine call
// (pydee.cpp:430-509).  This module keeps those method names, argument
// order and checks (expert_ids [tokens, topk] int32 on the host, topk equal
// to EngineConfig.topk, bool results with the reason in
// last_error_message()), so a caller swaps the import.  Everything below is
// a thin shim over include/dee_b200.h; the module links the in-tree
// libdee_b200.so and holds no CUDA code of its own.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "dee_b200.h"

namespace py = pybind11;

namespace {

class Engine {
public:
    Engine() = default;
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;
    ~Engine() { close(); }

    // Engine::init(EngineConfig) -> bool
    bool init(const dee_config& cfg) {
        close();
        cfg_ = cfg;
        dee_engine* e = nullptr;
        const int rc = dee_engine_create(&cfg, &e);
        if (rc != DEE_OK) {
            error_ = "dee_engine_create failed (status " + std::to_string(rc) + ")";
            return false;
        }
        engine_ = e;
        error_.clear();
        return true;
    }

    void close() {
        if (engine_) dee_engine_destroy(engine_);
        engine_ = nullptr;
    }

    const dee_config& config() const { return cfg_; }

    std::string last_error_message() const {
        if (!error_.empty()) return error_;
        return engine_ ? std::string(dee_last_error(engine_)) : std::string("engine not initialised");
    }

    // The expert records of one layer (device memory, DEE4 layout).
    bool attach_bank(int layer, uintptr_t d_records_ptr, int n_slots, size_t record_bytes) {
        if (!ready()) return false;
        int rc;
        {
            py::gil_scoped_release release;
            rc = dee_expert_bank_attach(engine_, layer, reinterpret_cast<const void*>(d_records_ptr), n_slots,
                                        record_bytes, nullptr);
        }
        return rc == DEE_OK;
    }

    bool moe_forward_batch_device(int layer, uintptr_t d_h_in_ptr, int tokens,
                                  py::array_t<int, py::array::c_style | py::array::forcecast> expert_ids,
                                  int topk, uintptr_t d_experts_out_ptr) {
        auto ids = expert_ids.request();
        if (ids.ndim != 2 || ids.shape[0] != tokens || ids.shape[1] != topk)
            throw std::runtime_error("expert_ids must have shape [tokens, topk]");
        if (topk != cfg_.topk) throw std::runtime_error("expert_ids topk does not match EngineConfig.topk");
        if (!ready()) return false;
        int rc;
        {
            py::gil_scoped_release release;
            rc = dee_moe_forward_batch_device(engine_, layer, reinterpret_cast<const void*>(d_h_in_ptr), tokens,
                                              static_cast<const int32_t*>(ids.ptr), topk,
                                              reinterpret_cast<void*>(d_experts_out_ptr));
        }
        return rc == DEE_OK;
    }

    bool moe_forward_combined_device(int layer, uintptr_t d_h_in_ptr, int tokens, uintptr_t d_expert_ids_ptr,
                                     int topk, uintptr_t d_weights_ptr, uintptr_t d_output_ptr,
                                     uintptr_t d_raw_trace_ptr, uintptr_t external_stream_ptr) {
        if (topk != cfg_.topk) throw std::runtime_error("expert_ids topk does not match EngineConfig.topk");
        if (!ready()) return false;
        int rc;
        {
            py::gil_scoped_release release;
            rc = dee_moe_forward_combined_device(
                engine_, layer, reinterpret_cast<const void*>(d_h_in_ptr), tokens,
                reinterpret_cast<const int64_t*>(d_expert_ids_ptr), topk,
                reinterpret_cast<const float*>(d_weights_ptr), reinterpret_cast<void*>(d_output_ptr),
                reinterpret_cast<void*>(d_raw_trace_ptr), reinterpret_cast<void*>(external_stream_ptr));
        }
        return rc == DEE_OK;
    }

    // dee_engine_sync_status: synchronise the stream, return (and clear) the
    // kernels' status word (0 = ok).
    uint32_t sync_status(uintptr_t stream_ptr) {
        if (!engine_) throw std::runtime_error("engine not initialised");
        uint32_t st = 0;
        int rc;
        {
            py::gil_scoped_release release;
            rc = dee_engine_sync_status(engine_, reinterpret_cast<void*>(stream_ptr), &st);
        }
        if (rc != DEE_OK && rc != DEE_ERR_DEVICE) throw std::runtime_error(last_error_message());
        return st;
    }

private:
    bool ready() {
        if (engine_) return true;
        error_ = "engine not initialised";
        return false;
    }

    dee_engine* engine_ = nullptr;
    dee_config cfg_{};
    std::string error_;
};

}  // namespace

PYBIND11_MODULE(_pydee, m) {
    m.doc() = "pydee.Engine's routed-expert methods over the dee_b200 C ABI (GIL released around engine calls)";
    m.def("abi_config_size", &dee_abi_config_size);

    py::class_<dee_config>(m, "EngineConfig")
        .def(py::init([](int hidden, int inter, int num_experts, int topk, int num_layers, int device_id,
                         float swiglu_limit, int max_tokens) {
                 dee_config c{};
                 c.hidden = hidden;
                 c.inter = inter;
                 c.num_experts = num_experts;
                 c.topk = topk;
                 c.num_layers = num_layers;
                 c.device_id = device_id;
                 c.swiglu_limit = swiglu_limit;
                 c.max_tokens = max_tokens;
                 return c;
             }),
             py::arg("hidden") = 4096, py::arg("inter") = 2048, py::arg("num_experts") = 256, py::arg("topk") = 6,
             py::arg("num_layers") = 1, py::arg("device_id") = 0, py::arg("swiglu_limit") = 0.0f,
             py::arg("max_tokens") = 64)
        .def_readwrite("hidden", &dee_config::hidden)
        .def_readwrite("inter", &dee_config::inter)
        .def_readwrite("num_experts", &dee_config::num_experts)
        .def_readwrite("topk", &dee_config::topk)
        .def_readwrite("num_layers", &dee_config::num_layers)
        .def_readwrite("device_id", &dee_config::device_id)
        .def_readwrite("swiglu_limit", &dee_config::swiglu_limit)
        .def_readwrite("max_tokens", &dee_config::max_tokens);

    py::class_<Engine>(m, "Engine")
        .def(py::init<>())
        .def("init", &Engine::init, py::arg("config"))
        .def("close", &Engine::close)
        .def("config", &Engine::config, py::return_value_policy::copy)
        .def("last_error_message", &Engine::last_error_message)
        .def("attach_bank", &Engine::attach_bank, py::arg("layer"), py::arg("d_records_ptr"), py::arg("n_slots"),
             py::arg("record_bytes"))
        .def("moe_forward_batch_device", &Engine::moe_forward_batch_device, py::arg("layer"),
             py::arg("d_h_in_ptr"), py::arg("tokens"), py::arg("expert_ids"), py::arg("topk"),
             py::arg("d_experts_out_ptr"),
             "FP16 hidden [tokens, H] on device, host int32 expert_ids [tokens, topk], FP32 raw expert "
             "outputs [tokens, topk, H] on device; synchronises the engine's stream; False on failure.")
        .def("moe_forward_combined_device", &Engine::moe_forward_combined_device, py::arg("layer"),
             py::arg("d_h_in_ptr"), py::arg("tokens"), py::arg("d_expert_ids_ptr"), py::arg("topk"),
             py::arg("d_weights_ptr"), py::arg("d_output_ptr"), py::arg("d_raw_trace_ptr"),
             py::arg("external_stream_ptr"),
             "Device int64 ids, FP32 weights, FP16 output combined in stable expert order, optional FP32 raw "
             "trace; queued on the caller's stream; False on failure.")
        .def("sync_status", &Engine::sync_status, py::arg("stream_ptr") = 0);
}
