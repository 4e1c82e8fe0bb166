// Drives the reference engine (its RuntimeBuilder, ExecutionPlanBuilder and
// Executor, compiled from its own sources) with the CUDA backend plugin of
// cuda_backend_plugin.cpp: the drop-in check of the kernel plugin boundary.
//
//   plugin_check resolve   (no GPU needed) -- the plugin's kernels are in the
//       reference's KernelRegistry under kCUDA selectors; a plan of kCUDA
//       RmsNorm / Add nodes resolves them through the plugin's Backend; a kCUDA
//       op the plugin does not provide fails with the registry's NotFound.
//   plugin_check execute   (GPU) -- the same plan runs through
//       Executor::Execute on device tensors: RMSNorm on the reference's unit
//       test inputs (tests/unit/backend/cpu/kernels/test_cpu_rmsnorm_kernel.cpp:
//       65-89 and 92-129) and a bf16 Add; prints the outputs.
// Exit code 0 = every check passed; messages on stdout.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "aethermind/backend/backend_factory.h"
#include "aethermind/execution/execution_plan_builder.h"
#include "aethermind/execution/executor.h"
#include "aethermind/execution/runtime_binding_context.h"
#include "aethermind/operators/operator_inference.h"
#include "aethermind/operators/rmsnorm_op.h"
#include "aethermind/runtime/runtime_builder.h"

extern "C" void* aethermind_b200_make_cuda_backend_factory();

using namespace aethermind;

namespace {

int g_fail = 0;
#define CHECK(cond, ...)                    \
    do {                                    \
        if (!(cond)) {                      \
            std::printf("FAIL: " __VA_ARGS__); \
            std::printf("\n");              \
            ++g_fail;                       \
        }                                   \
    } while (0)

SymbolicShape Shape(std::initializer_list<int64_t> dims) {
    return SymbolicShape(IntArrayView{std::vector<int64_t>(dims)});
}

RuntimeContext MakeRuntime() {
    RuntimeBuilder builder;
    builder.RegisterBackendFactory(DeviceType::kCUDA, std::unique_ptr<BackendFactory>(static_cast<BackendFactory*>(
                                                              aethermind_b200_make_cuda_backend_factory())));
    return builder.Build();
}

ExecutionPlanNodeSpec RmsNormNode(DataType dt, int64_t rows, int64_t hidden) {
    std::vector<TensorSpec> in = {TensorSpec{.dtype = dt, .shape = Shape({rows, hidden})},
                                  TensorSpec{.dtype = dt, .shape = Shape({hidden})}};
    const auto inferred = InferOperator(OpType::kRmsNorm, OpParams{RmsNormParams{.eps = 1.0e-5F}}, in);
    CHECK(inferred.ok(), "InferOperator(RmsNorm): %s", inferred.status().ToString().c_str());
    ExecutionPlanNodeSpec n{.op_type = OpType::kRmsNorm,
                            .device_type = DeviceType::kCUDA,
                            .act_dtype = dt,
                            .weight_dtype = dt,
                            .weight_format = WeightFormat::kPlain,
                            .isa = IsaLevel::kScalar,
                            .phase = ExecPhase::kBoth};
    n.input_specs = in;
    if (inferred.ok()) {
        n.output_specs = inferred->outputs;
        n.runtime_checks = inferred->runtime_checks;
    }
    n.op_params = OpParams{RmsNormParams{.eps = 1.0e-5F}};
    return n;
}

ExecutionPlanNodeSpec AddNode(DataType dt, int64_t count) {
    std::vector<TensorSpec> in = {TensorSpec{.dtype = dt, .shape = Shape({count})},
                                  TensorSpec{.dtype = dt, .shape = Shape({count})}};
    const auto inferred = InferOperator(OpType::kAdd, OpParams{AddParams{}}, in);
    CHECK(inferred.ok(), "InferOperator(Add): %s", inferred.status().ToString().c_str());
    ExecutionPlanNodeSpec n{.op_type = OpType::kAdd,
                            .device_type = DeviceType::kCUDA,
                            .act_dtype = dt,
                            .weight_dtype = dt,
                            .weight_format = WeightFormat::kPlain,
                            .isa = IsaLevel::kScalar,
                            .phase = ExecPhase::kBoth};
    n.input_specs = in;
    if (inferred.ok()) {
        n.output_specs = inferred->outputs;
        n.runtime_checks = inferred->runtime_checks;
    }
    n.op_params = OpParams{AddParams{}};
    return n;
}

int Resolve() {
    RuntimeContext rt = MakeRuntime();
    const std::vector<ExecutionPlanNodeSpec> nodes = {RmsNormNode(DataType::Float32(), 2, 4),
                                                      RmsNormNode(DataType::BFloat(16), 2, 4),
                                                      AddNode(DataType::BFloat(16), 8)};
    const auto plan = ExecutionPlanBuilder::Build(rt, nodes);
    CHECK(plan.ok(), "ExecutionPlanBuilder::Build: %s", plan.status().ToString().c_str());
    if (plan.ok()) {
        const char* want[3] = {"aethermind_b200::rmsnorm_cuda_f32", "aethermind_b200::rmsnorm_cuda_bf16",
                               "aethermind_b200::add_cuda_bf16"};
        CHECK(plan->size() == 3, "plan has %zu steps", plan->size());
        for (size_t i = 0; i < plan->size() && i < 3; ++i) {
            const ResolvedKernel& rk = plan->steps()[i].op->GetResolvedKernel();
            std::printf("step %zu: %s\n", i, rk.debug_name ? rk.debug_name : "(null)");
            CHECK(rk.debug_name && std::string(rk.debug_name) == want[i], "step %zu resolved %s", i,
                  rk.debug_name ? rk.debug_name : "(null)");
            CHECK(plan->steps()[i].selector.device_type == DeviceType::kCUDA, "step %zu not on kCUDA", i);
        }
    }
    // a kCUDA op this plugin does not provide: the registry says NotFound at plan time
    ExecutionPlanNodeSpec bad = RmsNormNode(DataType::Float32(), 2, 4);
    bad.isa = IsaLevel::kScalar;
    bad.act_dtype = bad.weight_dtype = DataType::Float32();
    bad.weight_format = WeightFormat::kQuantizedInt8;
    const auto p2 = ExecutionPlanBuilder::Build(rt, std::vector<ExecutionPlanNodeSpec>{bad});
    CHECK(!p2.ok(), "an unregistered kCUDA selector resolved");
    if (!p2.ok()) std::printf("unregistered selector: %s\n", p2.status().ToString().c_str());
    return g_fail == 0 ? 0 : 1;
}

uint16_t ToBf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float FromBf16(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int Execute() {
    RuntimeContext rt = MakeRuntime();
    const std::vector<ExecutionPlanNodeSpec> nodes = {RmsNormNode(DataType::Float32(), 2, 4),
                                                      AddNode(DataType::BFloat(16), 8)};
    auto plan = ExecutionPlanBuilder::Build(rt, nodes);
    CHECK(plan.ok(), "ExecutionPlanBuilder::Build: %s", plan.status().ToString().c_str());
    if (!plan.ok()) return 1;
    // RMSNorm rows: [1,2,3,4] with weight ones (golden row 0) and the same row
    // with weight [1, .5, 1.5, 2] computed as a second weight run below
    const float x[8] = {1.f, 2.f, 3.f, 4.f, 1.f, 2.f, 3.f, 4.f};
    const float w1[4] = {1.f, 1.f, 1.f, 1.f};
    float *dx = nullptr, *dw = nullptr, *dy = nullptr;
    uint16_t *da = nullptr, *db = nullptr, *dc = nullptr;
    cudaMalloc(&dx, sizeof x);
    cudaMalloc(&dw, sizeof w1);
    cudaMalloc(&dy, sizeof x);
    cudaMalloc(&da, 16);
    cudaMalloc(&db, 16);
    cudaMalloc(&dc, 16);
    cudaMemcpy(dx, x, sizeof x, cudaMemcpyHostToDevice);
    cudaMemcpy(dw, w1, sizeof w1, cudaMemcpyHostToDevice);
    uint16_t ha[8], hb[8];
    for (int i = 0; i < 8; ++i) {
        ha[i] = ToBf16(1.0f + 0.25f * (float)i);
        hb[i] = ToBf16(0.5f - 0.125f * (float)i);
    }
    cudaMemcpy(da, ha, 16, cudaMemcpyHostToDevice);
    cudaMemcpy(db, hb, 16, cudaMemcpyHostToDevice);
    const int64_t io_shape[2] = {2, 4}, io_str[2] = {4, 1}, w_shape[1] = {4}, w_str[1] = {1};
    const int64_t v_shape[1] = {8}, v_str[1] = {1};
    RuntimeBindingContext bindings;
    bindings.SetStepTensorBinding(
            0, StepTensorBinding{.inputs = {TensorView{dx, DataType::Float32(), io_shape, io_str},
                                            TensorView{dw, DataType::Float32(), w_shape, w_str}},
                                 .outputs = {MutableTensorView{dy, DataType::Float32(), io_shape, io_str}}});
    bindings.SetStepTensorBinding(
            1, StepTensorBinding{.inputs = {TensorView{da, DataType::BFloat(16), v_shape, v_str},
                                            TensorView{db, DataType::BFloat(16), v_shape, v_str}},
                                 .outputs = {MutableTensorView{dc, DataType::BFloat(16), v_shape, v_str}}});
    Status st = Executor::Execute(*plan, bindings);
    CHECK(st.ok(), "Executor::Execute: %s", st.ToString().c_str());
    CHECK(cudaDeviceSynchronize() == cudaSuccess, "device sync");
    float y[8];
    cudaMemcpy(y, dy, sizeof y, cudaMemcpyDeviceToHost);
    const float golden0[4] = {0.365148f, 0.730297f, 1.095445f, 1.460593f};
    std::printf("rmsnorm:");
    for (int i = 0; i < 8; ++i) std::printf(" %.6f", y[i]);
    std::printf("\n");
    for (int r = 0; r < 2; ++r)
        for (int i = 0; i < 4; ++i)
            CHECK(std::fabs(y[r * 4 + i] - golden0[i]) < 1e-5f, "rmsnorm[%d][%d] = %f, golden %f", r, i, y[r * 4 + i],
                  golden0[i]);
    // second golden: weight [1, .5, 1.5, 2] (test_cpu_rmsnorm_kernel.cpp:126-129), a fresh plan run
    const float w2[4] = {1.f, 0.5f, 1.5f, 2.f};
    cudaMemcpy(dw, w2, sizeof w2, cudaMemcpyHostToDevice);
    st = Executor::Execute(*plan, bindings);
    CHECK(st.ok() && cudaDeviceSynchronize() == cudaSuccess, "second Execute");
    cudaMemcpy(y, dy, sizeof y, cudaMemcpyDeviceToHost);
    const float golden1[4] = {0.365148f, 0.365148f, 1.643168f, 2.921186f};
    for (int i = 0; i < 4; ++i)
        CHECK(std::fabs(y[i] - golden1[i]) < 1e-5f, "rmsnorm w2[%d] = %f, golden %f", i, y[i], golden1[i]);
    uint16_t hc[8];
    cudaMemcpy(hc, dc, 16, cudaMemcpyDeviceToHost);
    std::printf("add:");
    for (int i = 0; i < 8; ++i) {
        const float want = FromBf16(ToBf16(FromBf16(ha[i]) + FromBf16(hb[i])));
        std::printf(" %.4f", FromBf16(hc[i]));
        CHECK(hc[i] == ToBf16(want), "add[%d] = %f, want %f", i, FromBf16(hc[i]), want);
    }
    std::printf("\n");
    cudaFree(dx);
    cudaFree(dw);
    cudaFree(dy);
    cudaFree(da);
    cudaFree(db);
    cudaFree(dc);
    return g_fail == 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "resolve";
    const int rc = mode == "execute" ? Execute() : Resolve();
    std::printf(rc == 0 ? "OK\n" : "FAILED (%d)\n", g_fail);
    return rc;
}
