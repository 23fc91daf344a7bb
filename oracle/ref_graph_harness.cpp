// Test-only harness: appended (on the compiler's stdin) after the reference's
// unmodified engine/src/executor.cpp so that the graph executor's static INT8
// activation quantiser (executor.cpp:220-230) and fused activations
// (executor.cpp:232-242), both in an anonymous namespace, can be called
// through a C ABI.  It is the reference oracle for the graph boundary
// and is never linked into the product.

#include <cstddef>
#include <cstdint>
#include <exception>
#include <string>

namespace {
thread_local std::string graph_harness_error;
}

extern "C" {

const char* leafref_graph_last_error() { return graph_harness_error.c_str(); }

// q[i] = nearbyint(clamp(x[i] / scale, -127, 127)); throws (returns 1) on a
// non-finite input or scale, exactly as the reference does.
int leafref_graph_quantize(const float* values, std::size_t count, float scale, std::int8_t* out) {
    try {
        const auto q = leaf::quantize_input(values, count, scale);
        for (std::size_t i = 0; i < count; ++i) out[i] = q[i];
        return 0;
    } catch (const std::exception& e) { graph_harness_error = e.what(); return 1; }
}

// out[i] = apply_activation(values[i], name): "", "Relu", "Silu" or "Gelu";
// an unknown name throws (returns 1), as the reference does.
int leafref_graph_activation(const float* values, std::size_t count, const char* name, float* out) {
    try {
        const std::string activation(name);
        for (std::size_t i = 0; i < count; ++i) out[i] = leaf::apply_activation(values[i], activation);
        return 0;
    } catch (const std::exception& e) { graph_harness_error = e.what(); return 1; }
}

}  // extern "C"
