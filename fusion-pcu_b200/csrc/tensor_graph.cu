// tensor_graph.cu -- host-side strict tensor graph: capture, reverse mode, plan and execution
// over the pcu_b200.h node kernels (host code only; see include/pcu_b200_graph.h for the
// reference files each part mirrors).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

#include "pcu_b200.h"
#include "pcu_b200_graph.h"
#include "provider.h"

namespace {

struct Node {
    int op = PCU_B200_NODE_INPUT;
    int32_t left = -1, right = -1;
    bool tl = false, tr = false;
    uint32_t rate_bits = 0;       // SgdUpdate learning rate (binary32)
    uint64_t scalar_bits = 0;     // Uniform value (element type bits)
    std::vector<uint64_t> shape;  // rank 0..2
    uint64_t count() const {
        uint64_t c = 1;
        for (uint64_t d : shape) c *= d;
        return c;
    }
};

bool is_checked(int op) {  // checked binary or strict compound: always planned (tensor.rs:3259-3271)
    return op == PCU_B200_NODE_ADD || op == PCU_B200_NODE_SUB || op == PCU_B200_NODE_MUL ||
           op == PCU_B200_NODE_DIV || op == PCU_B200_NODE_MATMUL || op == PCU_B200_NODE_MEAN_SQUARED_ERROR ||
           op == PCU_B200_NODE_SGD_UPDATE;
}

void clear(pcu_b200_tensor_error *e) {
    if (!e) return;
    std::memset(e, 0, sizeof(*e));
    e->value = -1;
}

int32_t fail(pcu_b200_tensor_error *e, int code, int32_t value = -1) {
    if (e) {
        clear(e);
        e->code = code;
        e->value = value;
    }
    return -1;
}

// exact binary32 -> binary64 widening (Crates/core/scalar_widen.rs:9-33)
uint64_t widen_f32_bits(uint32_t bits) {
    uint64_t sign = (uint64_t)(bits >> 31) << 63;
    uint32_t field = (bits >> 23) & 0xffu, frac = bits & 0x7fffffu;
    if (field == 0xffu) return sign | (0x7ffull << 52) | ((uint64_t)frac << 29);
    if (field) return sign | ((uint64_t)(field + 1023 - 127) << 52) | ((uint64_t)frac << 29);
    if (!frac) return sign;
    int lead = 31 - __builtin_clz(frac);
    uint64_t sig = (uint64_t)frac << (52 - lead);
    return sign | ((uint64_t)(lead + 874) << 52) | (sig & 0x000fffffffffffffull);
}

// count -> binary32/binary64 nearest-even bits (constants/constants.rs:18-27)
uint64_t count_bits(uint64_t n, bool f64) {
    const int frac = f64 ? 52 : 23, bias = f64 ? 1023 : 127;
    if (!n) return 0;
    int e = 63 - __builtin_clzll(n);
    uint64_t sig;
    if (e <= frac) {
        sig = n << (frac - e);
    } else {
        int sh = e - frac;
        uint64_t q = n >> sh, rem = n & ((1ull << sh) - 1), half = 1ull << (sh - 1);
        sig = q + (uint64_t)(rem > half || (rem == half && (q & 1)));
    }
    if (sig == (1ull << (frac + 1))) {
        sig >>= 1;
        e += 1;
    }
    return ((uint64_t)(e + bias) << frac) | (sig & ((1ull << frac) - 1));
}

// Checked 2 / count for the MSE gradient scale, evaluated at capture (gradients.rs:156-164).
// 2/count is exact or normal for every count a tensor can have, so the only possible fault of
// the reference's checked divide (underflow of a huge count) cannot occur below 2^126 elements.
uint64_t two_over_count_bits(uint64_t n, bool f64) {
    if (f64) {
        double c;
        uint64_t cb = count_bits(n, true);
        std::memcpy(&c, &cb, 8);
        double r = 2.0 / c;  // IEEE division, correctly rounded on the host
        uint64_t rb;
        std::memcpy(&rb, &r, 8);
        return rb;
    }
    float c;
    uint32_t cb = (uint32_t)count_bits(n, false);
    std::memcpy(&c, &cb, 4);
    float r = 2.0f / c;
    uint32_t rb;
    std::memcpy(&rb, &r, 4);
    return rb;
}

}  // namespace

struct pcu_b200_graph {
    int dtype = PCU_B200_F32;
    int policy = 0;
    std::vector<Node> nodes;

    bool valid(int32_t v) const { return v >= 0 && (size_t)v < nodes.size(); }
    int32_t push(Node n) {
        nodes.push_back(std::move(n));
        return (int32_t)nodes.size() - 1;
    }
    bool f64() const { return dtype == PCU_B200_F64; }
    uint64_t one_bits() const { return f64() ? 0x3ff0000000000000ull : 0x3f800000ull; }
    uint64_t minus_one_bits() const { return f64() ? 0xbff0000000000000ull : 0xbf800000ull; }

    int32_t binary(int op, int32_t a, int32_t b, pcu_b200_tensor_error *e) {
        if (!valid(a)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, a);
        if (!valid(b)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, b);
        if (nodes[a].shape != nodes[b].shape) return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH, b);
        Node n;
        n.op = PCU_B200_NODE_ADD + op;
        n.left = a;
        n.right = b;
        n.shape = nodes[a].shape;
        return push(std::move(n));
    }
    int32_t uniform(std::vector<uint64_t> shape, uint64_t bits) {
        Node n;
        n.op = PCU_B200_NODE_UNIFORM;
        n.shape = std::move(shape);
        n.scalar_bits = bits;
        return push(std::move(n));
    }
    int32_t matmul(int32_t a, int32_t b, bool tl, bool tr, pcu_b200_tensor_error *e) {
        if (!valid(a)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, a);
        if (!valid(b)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, b);
        const auto &sa = nodes[a].shape, &sb = nodes[b].shape;
        if (sa.size() != 2 || sb.size() != 2) return fail(e, PCU_B200_TENSOR_MATMUL_SHAPE, b);
        uint64_t rows = tl ? sa[1] : sa[0], inner = tl ? sa[0] : sa[1];
        uint64_t inner2 = tr ? sb[1] : sb[0], cols = tr ? sb[0] : sb[1];
        if (inner != inner2) return fail(e, PCU_B200_TENSOR_MATMUL_SHAPE, b);
        Node n;
        n.op = PCU_B200_NODE_MATMUL;
        n.left = a;
        n.right = b;
        n.tl = tl;
        n.tr = tr;
        n.shape = {rows, cols};
        return push(std::move(n));
    }
    int32_t relu_backward(int32_t x, int32_t up, pcu_b200_tensor_error *e) {
        if (!valid(x)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, x);
        if (!valid(up)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, up);
        if (nodes[x].shape != nodes[up].shape) return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH, up);
        Node n;
        n.op = PCU_B200_NODE_RELU_BACKWARD;
        n.left = x;
        n.right = up;
        n.shape = nodes[x].shape;
        return push(std::move(n));
    }

    // ---- reverse mode for an MSE root and one target (gradients.rs:31-444)
    void accumulate(std::vector<int32_t> &grads, int32_t target, int32_t addition) {
        grads[target] = grads[target] < 0 ? addition : binary(PCU_B200_ADD, grads[target], addition, nullptr);
    }

    // append_mse_gradients (gradients.rs:139-200): scale = 2/count as a Uniform of the
    // prediction's shape, then (p - t) * scale and/or (t - p) * scale
    void mse_gradient(std::vector<int32_t> &grads, int32_t prediction, int32_t tgt, const std::vector<bool> &needed) {
        if (!needed[prediction] && !needed[tgt]) return;
        int32_t scale = uniform(nodes[prediction].shape, two_over_count_bits(nodes[prediction].count(), f64()));
        int32_t pd = needed[prediction] ? binary(PCU_B200_SUB, prediction, tgt, nullptr) : -1;
        int32_t td = needed[tgt] ? binary(PCU_B200_SUB, tgt, prediction, nullptr) : -1;
        int32_t pg = pd >= 0 ? binary(PCU_B200_MUL, pd, scale, nullptr) : -1;
        int32_t tg = td >= 0 ? binary(PCU_B200_MUL, td, scale, nullptr) : -1;
        if (pg >= 0) accumulate(grads, prediction, pg);
        if (tg >= 0) accumulate(grads, tgt, tg);
    }

    // backward_mse_for_targets (gradients.rs:289-303 over build_backward_mse, :366-444): one shared
    // reverse sweep; out[j] receives d loss / d targets[j].  Returns 0 or -1 with *e filled.
    int32_t gradients(int32_t loss, const int32_t *targets, int count, int32_t *out, pcu_b200_tensor_error *e) {
        if (count <= 0 || !targets || !out) return fail(e, PCU_B200_TENSOR_EMPTY_OUTPUTS);
        for (int j = 0; j < count; ++j)
            if (!valid(targets[j])) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, targets[j]);
        if (!valid(loss)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, loss);
        if (nodes[loss].op != PCU_B200_NODE_MEAN_SQUARED_ERROR) return fail(e, PCU_B200_TENSOR_GRADIENT_ROOT_NOT_MSE, loss);
        const size_t original = nodes.size();
        // derivative_dependencies (gradients.rs:306-364): validate the loss closure, then mark
        // the values that depend on a requested target
        std::vector<bool> visited(original, false);
        std::vector<int32_t> pending{loss};
        while (!pending.empty()) {
            int32_t i = pending.back();
            pending.pop_back();
            if (visited[i]) continue;
            visited[i] = true;
            const Node &n = nodes[i];
            if ((i != loss && n.op == PCU_B200_NODE_MEAN_SQUARED_ERROR) || n.op == PCU_B200_NODE_DIV ||
                n.op == PCU_B200_NODE_RELU_BACKWARD)
                return fail(e, PCU_B200_TENSOR_UNSUPPORTED_GRADIENT, i);
            if (n.left >= 0) pending.push_back(n.left);
            if (n.right >= 0) pending.push_back(n.right);
        }
        std::vector<bool> needed(original, false);
        bool wants_loss = false;
        for (int j = 0; j < count; ++j) {
            if (!visited[targets[j]]) return fail(e, PCU_B200_TENSOR_UNSUPPORTED_GRADIENT, targets[j]);
            needed[targets[j]] = true;
            wants_loss |= targets[j] == loss;
        }
        for (int32_t i = 0; i <= loss; ++i) {
            const Node &n = nodes[i];
            if ((n.left >= 0 && needed[n.left]) || (n.right >= 0 && needed[n.right])) needed[i] = true;
        }
        std::vector<int32_t> grads(original, -1);
        if (wants_loss)  // d loss / d loss exposes the root cotangent, an exact Uniform(1)
            grads[loss] = uniform({}, one_bits());
        else
            mse_gradient(grads, nodes[loss].left, nodes[loss].right, needed);
        for (int32_t i = loss; i >= 0; --i) {
            const int32_t g = grads[i];
            if (g < 0) continue;
            const Node n = nodes[i];  // copy: appends may reallocate
            switch (n.op) {
            case PCU_B200_NODE_INPUT:
            case PCU_B200_NODE_UNIFORM:
                break;
            case PCU_B200_NODE_ADD:
                if (needed[n.left]) accumulate(grads, n.left, g);
                if (needed[n.right]) accumulate(grads, n.right, g);
                break;
            case PCU_B200_NODE_SUB:
                if (needed[n.left]) accumulate(grads, n.left, g);
                if (needed[n.right]) {
                    int32_t neg = uniform(nodes[n.right].shape, minus_one_bits());
                    accumulate(grads, n.right, binary(PCU_B200_MUL, g, neg, nullptr));
                }
                break;
            case PCU_B200_NODE_MUL: {
                int32_t lg = needed[n.left] ? binary(PCU_B200_MUL, g, n.right, nullptr) : -1;
                int32_t rg = needed[n.right] ? binary(PCU_B200_MUL, g, n.left, nullptr) : -1;
                if (lg >= 0) accumulate(grads, n.left, lg);
                if (rg >= 0) accumulate(grads, n.right, rg);
                break;
            }
            case PCU_B200_NODE_MATMUL: {
                int32_t lg = -1, rg = -1;
                if (needed[n.left])
                    lg = n.tl ? matmul(n.right, g, n.tr, true, nullptr) : matmul(g, n.right, false, !n.tr, nullptr);
                if (needed[n.right])
                    rg = n.tr ? matmul(g, n.left, true, n.tl, nullptr) : matmul(n.left, g, !n.tl, false, nullptr);
                if (lg >= 0) accumulate(grads, n.left, lg);
                if (rg >= 0) accumulate(grads, n.right, rg);
                break;
            }
            case PCU_B200_NODE_RELU:
                if (needed[n.left]) accumulate(grads, n.left, relu_backward(n.left, g, nullptr));
                break;
            case PCU_B200_NODE_MEAN_SQUARED_ERROR:  // only the root: nested MSE was rejected above
                mse_gradient(grads, n.left, n.right, needed);
                break;
            case PCU_B200_NODE_SGD_UPDATE: {
                int32_t ig = -1;
                if (needed[n.right]) {
                    const uint32_t neg_rate = n.rate_bits ^ 0x80000000u;
                    int32_t scaled = uniform(nodes[n.right].shape, f64() ? widen_f32_bits(neg_rate) : neg_rate);
                    ig = binary(PCU_B200_MUL, g, scaled, nullptr);
                }
                if (needed[n.left]) accumulate(grads, n.left, g);
                if (ig >= 0) accumulate(grads, n.right, ig);
                break;
            }
            default:
                return fail(e, PCU_B200_TENSOR_UNSUPPORTED_GRADIENT, i);
            }
        }
        for (int j = 0; j < count; ++j) {
            if (grads[targets[j]] < 0) return fail(e, PCU_B200_TENSOR_UNSUPPORTED_GRADIENT, targets[j]);
            out[j] = grads[targets[j]];
        }
        clear(e);
        return 0;
    }
};

// ============================================================================ execution
struct pcu_b200_prepared {
    pcu_b200_graph graph;           // frozen copy of the captured graph
    std::vector<int32_t> plan;      // node ids in graph order
    std::vector<int32_t> inputs;    // planned Input node ids in capture order
    std::vector<void *> buffers;    // per node id (nullptr if not planned)
    uint64_t *status = nullptr;     // per node id
    uint64_t *disp = nullptr;       // per node id: guarded-chain disposition (pending 0, executed 1, skipped 2)
    std::vector<int32_t> stages;    // the planned nodes that launch work, in plan order
    // Per stage: how many of the stages right after a MatMul run in its epilogue in the chained
    // mode (pcu_b200_strict_matmul_epilogue); 0 for every other stage.
    std::vector<int> fused;
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    size_t elem = 4;
    cudaGraphExec_t replay = nullptr;  // the node launches recorded as one CUDA graph
    cudaStream_t replay_stream = nullptr;  // the stream it was recorded on
    cudaStream_t own_stream = nullptr;     // used for replay when the caller passes the legacy stream
    ~pcu_b200_prepared() {
        if (replay) cudaGraphExecDestroy(replay);
        if (own_stream) cudaStreamDestroy(own_stream);
        for (void *b : buffers)
            if (b) cudaFree(b);
        if (status) cudaFree(status);
        if (disp) cudaFree(disp);
        if (workspace) cudaFree(workspace);
    }
};

namespace {

int backend_error(pcu_b200_tensor_error *e, int32_t value, int code) {
    fail(e, PCU_B200_TENSOR_BACKEND, value);
    if (e) e->backend = code;
    return PCU_B200_TENSOR_BACKEND;
}

// Decode node `id`'s status word into the reference's TensorError (0 = no fault).
int decode(const pcu_b200_prepared &p, int32_t id, uint64_t word, pcu_b200_tensor_error *e) {
    if (word == PCU_B200_STATUS_OK) return 0;
    const Node &n = p.graph.nodes[id];
    const uint64_t event = word >> 3;
    const int kind = (int)(word & 7);
    if (kind < 1 || kind > 5) return backend_error(e, id, kind == PCU_B200_STATUS_WATCHDOG ? -7 : -1);
    clear(e);
    e->value = id;
    e->kind = kind;
    switch (n.op) {
    case PCU_B200_NODE_MATMUL: {
        const auto &sa = p.graph.nodes[n.left].shape;
        const uint64_t inner = n.tl ? sa[0] : sa[1];
        const uint64_t pair = event / 2;
        e->code = PCU_B200_TENSOR_COMPOUND_ARITHMETIC_FAULT;
        e->element_index = pair / inner;
        e->reduction_index = pair % inner;
        e->step = (event % 2) ? PCU_B200_STEP_ADD : PCU_B200_STEP_MULTIPLY;
        if (e->element_index >= n.count()) return backend_error(e, id, -1);
        break;
    }
    case PCU_B200_NODE_SGD_UPDATE:
        e->code = PCU_B200_TENSOR_COMPOUND_ARITHMETIC_FAULT;
        e->element_index = event / 2;
        e->reduction_index = 0;
        e->step = (event % 2) ? PCU_B200_STEP_SUBTRACT : PCU_B200_STEP_MULTIPLY;
        break;
    case PCU_B200_NODE_MEAN_SQUARED_ERROR: {
        const uint64_t count = p.graph.nodes[n.left].count();
        e->code = PCU_B200_TENSOR_COMPOUND_ARITHMETIC_FAULT;
        e->element_index = 0;
        if (event == 3 * count) {
            e->reduction_index = count;
            e->step = PCU_B200_STEP_DIVIDE;
        } else {
            e->reduction_index = event / 3;
            const int steps[3] = {PCU_B200_STEP_SUBTRACT, PCU_B200_STEP_MULTIPLY, PCU_B200_STEP_ADD};
            e->step = steps[event % 3];
        }
        break;
    }
    default:
        e->code = PCU_B200_TENSOR_ARITHMETIC_FAULT;
        e->element_index = event;
        break;
    }
    return e->code;
}

// The epilogue form of MatMul stage i with its p.fused[i] following stages.
int launch_fused(pcu_b200_prepared &p, size_t i, void *stream) {
    const int32_t id = p.stages[i];
    const Node &n = p.graph.nodes[id];
    pcu_b200_epilogue_stage st[PCU_B200_EPILOGUE_MAX] = {};
    int32_t value = id;  // the node whose result the next stage takes
    for (int k = 0; k < p.fused[i]; ++k) {
        const int32_t sid = p.stages[i + 1 + k];
        const Node &f = p.graph.nodes[sid];
        if (f.op == PCU_B200_NODE_RELU) {
            st[k].op = PCU_B200_EPILOGUE_RELU;
        } else {
            const bool value_left = f.left == value;
            const int32_t other = value_left ? f.right : f.left;
            st[k].op = f.op == PCU_B200_NODE_RELU_BACKWARD ? PCU_B200_EPILOGUE_RELU_BACKWARD : f.op - PCU_B200_NODE_ADD;
            st[k].operand = p.buffers[other];
            st[k].operand_uniform = p.graph.nodes[other].op == PCU_B200_NODE_UNIFORM ? 1 : 0;
            st[k].operand_left = value_left ? 0 : 1;
        }
        st[k].out = p.buffers[sid];
        st[k].status = p.status + sid;
        value = sid;
    }
    const auto &sa = p.graph.nodes[n.left].shape, &sb = p.graph.nodes[n.right].shape;
    const uint64_t inner = n.tl ? sa[0] : sa[1];
    return pcu::strict_matmul(p.graph.dtype, p.graph.policy, p.buffers[n.left], p.buffers[n.right], p.buffers[id],
                              n.shape[0], inner, n.shape[1], sa[1], sb[1], n.tl, n.tr, p.workspace, p.workspace_bytes,
                              p.status + id, stream, pcu::ChainGuard{}, st, p.fused[i]);
}

// Which stages the chained mode runs in a MatMul's epilogue: up to PCU_B200_EPILOGUE_MAX stages
// right after it in plan order, each an elementwise node (checked Add/Sub/Mul/Div, ReLU,
// ReLU-backward) of the same shape that takes the previous stage's result as exactly one of its
// operands.  The stages are consecutive, so the first faulting node in graph order is the same
// as when they run one by one.
void plan_fusion(pcu_b200_prepared &p) {
    const auto &nodes = p.graph.nodes;
    p.fused.assign(p.stages.size(), 0);
    for (size_t i = 0; i < p.stages.size(); ++i) {
        const Node &m = nodes[p.stages[i]];
        if (m.op != PCU_B200_NODE_MATMUL || m.count() == 0) continue;
        int32_t value = p.stages[i];
        int k = 0;
        while (k < PCU_B200_EPILOGUE_MAX && i + 1 + k < p.stages.size()) {
            const Node &f = nodes[p.stages[i + 1 + k]];
            bool ok = f.shape == m.shape;
            if (f.op == PCU_B200_NODE_RELU) {
                ok = ok && f.left == value;
            } else if ((f.op >= PCU_B200_NODE_ADD && f.op <= PCU_B200_NODE_DIV) || f.op == PCU_B200_NODE_RELU_BACKWARD) {
                ok = ok && ((f.left == value) != (f.right == value));
                const int32_t other = f.left == value ? f.right : f.left;
                ok = ok && other >= 0 && nodes[other].shape == m.shape && p.buffers[other];
            } else {
                ok = false;
            }
            if (!ok) break;
            value = p.stages[i + 1 + k];
            ++k;
        }
        p.fused[i] = k;
        i += k;
    }
}

int launch(pcu_b200_prepared &p, int32_t id, void *stream, const pcu::ChainGuard &guard) {
    const Node &n = p.graph.nodes[id];
    const int dt = p.graph.dtype, pol = p.graph.policy;
    uint64_t *st = p.status + id;
    void *out = p.buffers[id];
    auto buf = [&](int32_t v) { return p.buffers[v]; };
    auto uni = [&](int32_t v) { return p.graph.nodes[v].op == PCU_B200_NODE_UNIFORM ? 1 : 0; };
    switch (n.op) {
    case PCU_B200_NODE_INPUT:
    case PCU_B200_NODE_UNIFORM:
        return PCU_B200_OK;
    case PCU_B200_NODE_ADD:
    case PCU_B200_NODE_SUB:
    case PCU_B200_NODE_MUL:
    case PCU_B200_NODE_DIV:
        return pcu::checked_binary(dt, pol, n.op - PCU_B200_NODE_ADD, buf(n.left), buf(n.right), out, n.count(),
                                   uni(n.left), uni(n.right), st, stream, guard);
    case PCU_B200_NODE_RELU:
        return pcu::checked_relu(dt, pol, buf(n.left), out, n.count(), st, stream, guard);
    case PCU_B200_NODE_RELU_BACKWARD:
        return pcu::checked_relu_backward(dt, pol, buf(n.left), buf(n.right), out, n.count(), st, stream, guard);
    case PCU_B200_NODE_MATMUL: {
        const auto &sa = p.graph.nodes[n.left].shape, &sb = p.graph.nodes[n.right].shape;
        const uint64_t inner = n.tl ? sa[0] : sa[1];
        return pcu::strict_matmul(dt, pol, buf(n.left), buf(n.right), out, n.shape[0], inner, n.shape[1], sa[1], sb[1],
                                  n.tl, n.tr, p.workspace, p.workspace_bytes, st, stream, guard);
    }
    case PCU_B200_NODE_MEAN_SQUARED_ERROR:
        return pcu::strict_mse(dt, pol, buf(n.left), buf(n.right), out, p.graph.nodes[n.left].count(), p.workspace,
                               p.workspace_bytes, st, stream, guard);
    case PCU_B200_NODE_SGD_UPDATE:
        return pcu::strict_sgd(dt, pol, buf(n.left), buf(n.right), out, n.count(), n.rate_bits, st, stream, guard);
    default:
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    }
}

}  // namespace

// ============================================================================ C ABI
extern "C" pcu_b200_graph *pcu_b200_graph_new(int dtype, int policy) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2) return nullptr;
    auto *g = new (std::nothrow) pcu_b200_graph;
    if (g) {
        g->dtype = dtype;
        g->policy = policy;
    }
    return g;
}

extern "C" void pcu_b200_graph_free(pcu_b200_graph *graph) { delete graph; }

static bool shape_of(const uint64_t *shape, int rank, std::vector<uint64_t> &out) {
    if (rank < 0 || rank > 2 || (rank > 0 && !shape)) return false;
    out.assign(shape, shape + rank);
    return true;
}

extern "C" int32_t pcu_b200_graph_input(pcu_b200_graph *g, const uint64_t *shape, int rank, pcu_b200_tensor_error *e) {
    Node n;
    if (!g || !shape_of(shape, rank, n.shape)) return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH);
    n.op = PCU_B200_NODE_INPUT;
    clear(e);
    return g->push(std::move(n));
}

extern "C" int32_t pcu_b200_graph_uniform(pcu_b200_graph *g, const uint64_t *shape, int rank, uint64_t bits,
                                          pcu_b200_tensor_error *e) {
    std::vector<uint64_t> s;
    if (!g || !shape_of(shape, rank, s)) return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH);
    clear(e);
    return g->uniform(std::move(s), bits);
}

extern "C" int32_t pcu_b200_graph_binary(pcu_b200_graph *g, int op, int32_t a, int32_t b, pcu_b200_tensor_error *e) {
    if (!g || op < 0 || op > 3) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE);
    int32_t v = g->binary(op, a, b, e);
    if (v >= 0) clear(e);
    return v;
}

extern "C" int32_t pcu_b200_graph_relu(pcu_b200_graph *g, int32_t x, pcu_b200_tensor_error *e) {
    if (!g || !g->valid(x)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, x);
    Node n;
    n.op = PCU_B200_NODE_RELU;
    n.left = x;
    n.shape = g->nodes[x].shape;
    clear(e);
    return g->push(std::move(n));
}

extern "C" int32_t pcu_b200_graph_relu_backward(pcu_b200_graph *g, int32_t x, int32_t up, pcu_b200_tensor_error *e) {
    if (!g) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE);
    int32_t v = g->relu_backward(x, up, e);
    if (v >= 0) clear(e);
    return v;
}

extern "C" int32_t pcu_b200_graph_matmul(pcu_b200_graph *g, int32_t a, int32_t b, int tl, int tr,
                                         pcu_b200_tensor_error *e) {
    if (!g) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE);
    int32_t v = g->matmul(a, b, tl != 0, tr != 0, e);
    if (v >= 0) clear(e);
    return v;
}

extern "C" int32_t pcu_b200_graph_mean_squared_error(pcu_b200_graph *g, int32_t p, int32_t t,
                                                     pcu_b200_tensor_error *e) {
    if (!g || !g->valid(p)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, p);
    if (!g->valid(t)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, t);
    if (g->nodes[p].shape != g->nodes[t].shape || g->nodes[p].count() == 0)
        return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH, t);
    Node n;
    n.op = PCU_B200_NODE_MEAN_SQUARED_ERROR;
    n.left = p;
    n.right = t;
    clear(e);
    return g->push(std::move(n));
}

extern "C" int32_t pcu_b200_graph_sgd_update(pcu_b200_graph *g, int32_t w, int32_t grad, uint32_t rate_bits,
                                             pcu_b200_tensor_error *e) {
    if (!g || !g->valid(w)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, w);
    if (!g->valid(grad)) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, grad);
    if (g->nodes[w].shape != g->nodes[grad].shape) return fail(e, PCU_B200_TENSOR_SHAPE_MISMATCH, grad);
    if ((rate_bits & 0x7f800000u) == 0x7f800000u) return fail(e, PCU_B200_TENSOR_INVALID_LEARNING_RATE);
    Node n;
    n.op = PCU_B200_NODE_SGD_UPDATE;
    n.left = w;
    n.right = grad;
    n.rate_bits = rate_bits;
    n.shape = g->nodes[w].shape;
    clear(e);
    return g->push(std::move(n));
}

extern "C" int32_t pcu_b200_graph_gradient(pcu_b200_graph *g, int32_t loss, int32_t target, pcu_b200_tensor_error *e) {
    if (!g) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE);
    int32_t out = -1;
    return g->gradients(loss, &target, 1, &out, e) == 0 ? out : -1;
}

extern "C" int pcu_b200_graph_gradients(pcu_b200_graph *g, int32_t loss, const int32_t *targets, int count,
                                        int32_t *gradients, pcu_b200_tensor_error *e) {
    if (!g) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE), PCU_B200_TENSOR_UNKNOWN_VALUE;
    return g->gradients(loss, targets, count, gradients, e) == 0 ? PCU_B200_TENSOR_OK : e ? e->code : -1;
}

extern "C" int32_t pcu_b200_graph_node_count(const pcu_b200_graph *g) { return g ? (int32_t)g->nodes.size() : 0; }

extern "C" int pcu_b200_graph_describe(const pcu_b200_graph *g, int32_t v, int32_t *op, int32_t *left, int32_t *right,
                                       int32_t *tl, int32_t *tr, uint64_t *shape, int32_t *rank,
                                       uint64_t *scalar_bits) {
    if (!g || !g->valid(v)) return PCU_B200_TENSOR_UNKNOWN_VALUE;
    const Node &n = g->nodes[v];
    if (op) *op = n.op;
    if (left) *left = n.left;
    if (right) *right = n.right;
    if (tl) *tl = n.tl;
    if (tr) *tr = n.tr;
    if (rank) *rank = (int32_t)n.shape.size();
    if (shape)
        for (size_t i = 0; i < n.shape.size(); ++i) shape[i] = n.shape[i];
    if (scalar_bits) *scalar_bits = n.op == PCU_B200_NODE_SGD_UPDATE ? n.rate_bits : n.scalar_bits;
    return 0;
}

extern "C" pcu_b200_prepared *pcu_b200_graph_prepare(const pcu_b200_graph *g, const int32_t *outputs, int count,
                                                     pcu_b200_tensor_error *e) {
    if (!g) {
        fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE);
        return nullptr;
    }
    if (count <= 0 || !outputs) {
        fail(e, PCU_B200_TENSOR_EMPTY_OUTPUTS);
        return nullptr;
    }
    std::unique_ptr<pcu_b200_prepared> p(new (std::nothrow) pcu_b200_prepared);
    if (!p) {
        fail(e, PCU_B200_TENSOR_BACKEND);
        return nullptr;
    }
    p->graph = *g;
    p->elem = g->dtype == PCU_B200_F64 ? 8 : 4;
    const size_t N = g->nodes.size();
    std::vector<bool> selected(N, false);
    auto close = [&](int32_t root) {
        std::vector<int32_t> stack{root};
        while (!stack.empty()) {
            int32_t at = stack.back();
            stack.pop_back();
            if (selected[at]) continue;
            selected[at] = true;
            if (g->nodes[at].left >= 0) stack.push_back(g->nodes[at].left);
            if (g->nodes[at].right >= 0) stack.push_back(g->nodes[at].right);
        }
    };
    for (int i = 0; i < count; ++i) {
        if (!g->valid(outputs[i])) {
            fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE, outputs[i]);
            return nullptr;
        }
        close(outputs[i]);
    }
    for (size_t i = 0; i < N; ++i)
        if (is_checked(g->nodes[i].op)) close((int32_t)i);
    p->buffers.assign(N, nullptr);
    size_t ws = 0;
    for (size_t i = 0; i < N; ++i) {
        if (!selected[i]) continue;
        const Node &n = g->nodes[i];
        p->plan.push_back((int32_t)i);
        if (n.op == PCU_B200_NODE_INPUT) p->inputs.push_back((int32_t)i);
        const size_t bytes = std::max<size_t>(n.count(), 1) * p->elem;
        cudaError_t err = cudaMalloc(&p->buffers[i], bytes);
        if (err != cudaSuccess) {
            backend_error(e, (int32_t)i, (int)err);
            return nullptr;
        }
        if (n.op == PCU_B200_NODE_UNIFORM) {  // constants are materialised once at preparation
            std::vector<unsigned char> host(bytes);
            for (uint64_t k = 0; k < std::max<uint64_t>(n.count(), 1); ++k)
                std::memcpy(host.data() + k * p->elem, &n.scalar_bits, p->elem);
            err = cudaMemcpy(p->buffers[i], host.data(), bytes, cudaMemcpyHostToDevice);
            if (err != cudaSuccess) {
                backend_error(e, (int32_t)i, (int)err);
                return nullptr;
            }
        }
        if (n.op == PCU_B200_NODE_MATMUL) {
            const auto &sa = g->nodes[n.left].shape;
            ws = std::max(ws, pcu_b200_strict_matmul_workspace_size(n.shape[0], n.tl ? sa[0] : sa[1], n.shape[1]));
        }
        if (n.op == PCU_B200_NODE_MEAN_SQUARED_ERROR)
            ws = std::max(ws, pcu_b200_strict_mse_workspace_size(g->dtype, g->nodes[n.left].count()));
    }
    for (int32_t id : p->plan)
        if (g->nodes[id].op != PCU_B200_NODE_INPUT && g->nodes[id].op != PCU_B200_NODE_UNIFORM) p->stages.push_back(id);
    plan_fusion(*p);
    cudaError_t err = cudaMalloc((void **)&p->status, std::max<size_t>(N, 1) * sizeof(uint64_t));
    if (err == cudaSuccess) err = cudaMalloc((void **)&p->disp, std::max<size_t>(N, 1) * sizeof(uint64_t));
    if (err == cudaSuccess && ws) err = cudaMalloc(&p->workspace, ws);
    if (err != cudaSuccess) {
        backend_error(e, -1, (int)err);
        return nullptr;
    }
    p->workspace_bytes = ws;
    clear(e);
    return p.release();
}

extern "C" void pcu_b200_prepared_free(pcu_b200_prepared *p) { delete p; }

extern "C" int32_t pcu_b200_prepared_input_count(const pcu_b200_prepared *p) { return p ? (int32_t)p->inputs.size() : 0; }

extern "C" int32_t pcu_b200_prepared_input_value(const pcu_b200_prepared *p, int32_t i) {
    return (p && i >= 0 && (size_t)i < p->inputs.size()) ? p->inputs[i] : -1;
}

extern "C" void *pcu_b200_prepared_buffer(const pcu_b200_prepared *p, int32_t v) {
    return (p && v >= 0 && (size_t)v < p->buffers.size()) ? p->buffers[v] : nullptr;
}

namespace {

// The guard of stage i: its predecessor's fault word and disposition, and its own disposition.
pcu::ChainGuard stage_guard(const pcu_b200_prepared &p, size_t i) {
    pcu::ChainGuard g{};
    const int32_t id = p.stages[i];
    g.disp = reinterpret_cast<unsigned long long *>(p.disp + id);
    g.decide = 1;
    if (i > 0) {
        g.prev_status = reinterpret_cast<const unsigned long long *>(p.status + p.stages[i - 1]);
        g.prev_disp = reinterpret_cast<const unsigned long long *>(p.disp + p.stages[i - 1]);
    }
    return g;
}

// The status reset and every planned node, launched back to back on `s`; `guarded`: as a
// guarded chain (dispositions reset to pending, each stage admitted by its predecessor).
int launch_plan(pcu_b200_prepared &p, cudaStream_t s, int32_t &failed, bool guarded) {
    failed = -1;
    int rc = pcu_b200_status_reset(p.status, p.graph.nodes.size(), s);
    if (rc) return rc;
    if (guarded) {
        cudaError_t err = cudaMemsetAsync(p.disp, 0, p.graph.nodes.size() * sizeof(uint64_t), s);
        if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
    }
    for (size_t i = 0; i < p.stages.size(); ++i) {
        // the chained mode runs fusable stages in their MatMul's epilogue; the guarded chain keeps
        // one kernel per stage (a skipped stage must touch nothing)
        if (!guarded && p.fused[i]) {
            rc = launch_fused(p, i, s);
            if (rc) {
                failed = p.stages[i];
                return rc;
            }
            i += p.fused[i];
            continue;
        }
        rc = launch(p, p.stages[i], s, guarded ? stage_guard(p, i) : pcu::ChainGuard{});
        if (rc) {
            failed = p.stages[i];
            return rc;
        }
    }
    return PCU_B200_OK;
}

// One read of every status word; the lowest faulting node in graph order wins.  A guarded
// chain's records are also validated as the reference does (guarded.rs:109-147): every stage in
// front of the first fault executed without a fault, every stage after it was skipped with a
// clear fault word, and none is pending.  A violation blocks the result (FailedCompletion).
int read_and_decode(pcu_b200_prepared &p, cudaStream_t s, pcu_b200_tensor_error *e, bool guarded) {
    const size_t N = p.graph.nodes.size();
    std::vector<uint64_t> words(N), disp(guarded ? N : 0);
    cudaError_t err = cudaMemcpyAsync(words.data(), p.status, N * 8, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess && guarded) err = cudaMemcpyAsync(disp.data(), p.disp, N * 8, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return backend_error(e, -1, (int)err);
    if (guarded) {
        int32_t first = -1;
        for (int32_t id : p.stages) {
            const bool executed = disp[id] == pcu::kDispExecuted, skipped = disp[id] == pcu::kDispSkipped;
            const bool ok = first < 0 ? executed : (skipped && words[id] == PCU_B200_STATUS_OK);
            if (!ok) {
                fail(e, PCU_B200_TENSOR_FAILED_COMPLETION, id);
                return PCU_B200_TENSOR_FAILED_COMPLETION;
            }
            if (first < 0 && words[id] != PCU_B200_STATUS_OK) first = id;
        }
        if (first >= 0) return decode(p, first, words[first], e);
        return PCU_B200_TENSOR_OK;
    }
    for (int32_t id : p.plan)
        if (int code = decode(p, id, words[id], e)) return code;
    return PCU_B200_TENSOR_OK;
}

// Record the launch sequence of the plan as a CUDA graph on `s` (after one ordinary run, so that
// every kernel's one-time host set-up has happened outside the capture).
int record_replay(pcu_b200_prepared &p, cudaStream_t s, pcu_b200_tensor_error *e) {
    cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return backend_error(e, -1, (int)err);
    int32_t failed = -1;
    const int rc = launch_plan(p, s, failed, true);
    cudaGraph_t g = nullptr;
    err = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return backend_error(e, failed, rc);
    }
    if (err != cudaSuccess) return backend_error(e, -1, (int)err);
    err = cudaGraphInstantiate(&p.replay, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) {
        p.replay = nullptr;
        return backend_error(e, -1, (int)err);
    }
    p.replay_stream = s;
    return PCU_B200_TENSOR_OK;
}

}  // namespace

extern "C" int pcu_b200_prepared_execute(pcu_b200_prepared *p, const void *const *host_inputs, int mode,
                                         void *stream, pcu_b200_tensor_error *e) {
    clear(e);
    if (!p) return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE), PCU_B200_TENSOR_UNKNOWN_VALUE;
    if (mode < PCU_B200_EXEC_CHAINED || mode > PCU_B200_EXEC_GUARDED)
        return fail(e, PCU_B200_TENSOR_UNKNOWN_VALUE), PCU_B200_TENSOR_UNKNOWN_VALUE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (mode == PCU_B200_EXEC_GRAPH && !s) {  // a CUDA graph cannot be recorded on the legacy stream
        if (!p->own_stream) {
            cudaError_t err = cudaStreamCreateWithFlags(&p->own_stream, cudaStreamNonBlocking);
            if (err != cudaSuccess) return backend_error(e, -1, (int)err);
        }
        s = p->own_stream;
    }
    for (size_t i = 0; i < p->inputs.size(); ++i) {
        if (!host_inputs || !host_inputs[i]) continue;
        const int32_t v = p->inputs[i];
        cudaError_t err = cudaMemcpyAsync(p->buffers[v], host_inputs[i], p->graph.nodes[v].count() * p->elem,
                                          cudaMemcpyHostToDevice, s);
        if (err != cudaSuccess) return backend_error(e, v, (int)err);
    }
    if (mode == PCU_B200_EXEC_GRAPH) {  // the guarded chain, replayed as one CUDA graph
        if (p->replay && p->replay_stream == s) {
            cudaError_t err = cudaGraphLaunch(p->replay, s);
            if (err != cudaSuccess) return backend_error(e, -1, (int)err);
            return read_and_decode(*p, s, e, true);
        }
        // first run on this stream: an ordinary run gives the answer, then the plan is recorded
        int32_t failed = -1;
        const int rc = launch_plan(*p, s, failed, true);
        if (rc) return backend_error(e, failed, rc);
        const int code = read_and_decode(*p, s, e, true);
        if (p->replay) {
            cudaGraphExecDestroy(p->replay);
            p->replay = nullptr;
        }
        pcu_b200_tensor_error scratch;
        const int rec = record_replay(*p, s, &scratch);
        if (rec && !code) {
            if (e) *e = scratch;
            return rec;
        }
        return code;
    }
    if (mode != PCU_B200_EXEC_EACH_NODE) {  // chained or guarded: one observation at the end
        const bool guarded = mode == PCU_B200_EXEC_GUARDED;
        int32_t failed = -1;
        const int rc = launch_plan(*p, s, failed, guarded);
        if (rc) return backend_error(e, failed, rc);
        return read_and_decode(*p, s, e, guarded);
    }
    int rc = pcu_b200_status_reset(p->status, p->graph.nodes.size(), stream);
    if (rc) return backend_error(e, -1, rc);
    uint64_t word = 0;
    for (int32_t id : p->stages) {
        rc = launch(*p, id, stream, pcu::ChainGuard{});
        if (rc) return backend_error(e, id, rc);
        // the reference's per-node completion wait and status decode (strict_matmul.rs:317-331)
        cudaError_t err = cudaMemcpyAsync(&word, p->status + id, 8, cudaMemcpyDeviceToHost, s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
        if (err != cudaSuccess) return backend_error(e, id, (int)err);
        if (int code = decode(*p, id, word, e)) return code;
    }
    return PCU_B200_TENSOR_OK;
}

extern "C" int pcu_b200_prepared_fused(const pcu_b200_prepared *p, int32_t value) {
    if (!p) return 0;
    for (size_t i = 0; i < p->stages.size(); ++i)
        if (p->stages[i] == value) return p->fused[i];
    return 0;
}

extern "C" int pcu_b200_prepared_stage(const pcu_b200_prepared *p, int32_t value, uint64_t *fault_word,
                                       uint64_t *disposition, void *stream) {
    if (!p || value < 0 || (size_t)value >= p->buffers.size() || !p->buffers[value])
        return PCU_B200_TENSOR_UNKNOWN_VALUE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t err = cudaSuccess;
    if (fault_word) err = cudaMemcpyAsync(fault_word, p->status + value, 8, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess && disposition)
        err = cudaMemcpyAsync(disposition, p->disp + value, 8, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    return err == cudaSuccess ? PCU_B200_TENSOR_OK : PCU_B200_TENSOR_BACKEND;
}

extern "C" int pcu_b200_prepared_read(const pcu_b200_prepared *p, int32_t v, void *host, size_t bytes, void *stream) {
    if (!p || v < 0 || (size_t)v >= p->buffers.size() || !p->buffers[v]) return PCU_B200_TENSOR_UNKNOWN_VALUE;
    const size_t need = std::max<uint64_t>(p->graph.nodes[v].count(), 1) * p->elem;
    if (bytes < need) return PCU_B200_TENSOR_DATA_LENGTH;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemcpyAsync(host, p->buffers[v], need, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    return err == cudaSuccess ? PCU_B200_TENSOR_OK : PCU_B200_TENSOR_BACKEND;
}
