// Native graph executor: the CUDA counterpart of ComputationalGraph.Execute
// (src/Lokad.Onnx.Backend/ComputationalGraph.cs:199-272) and Node.ExecuteCPU
// (src/Lokad.Onnx.Backend/Node.cs:121-181).
//
// Nodes run in file order; tensors are resolved by name from inputs,
// initializers and intermediate outputs.  Float tensors live on the device
// for their whole life; small int64 tensors (shapes, axes) live on the host
// and are uploaded only when a kernel reads them (Gather indices, Cast).
// Every op is an asynchronous launch on the context's single stream; nothing
// synchronises until an output is read.
//
// lonnx_graph_prepare(g, flags) runs a pattern-fusion pass (flags & 1):
//   MatMul(x, W) -> Add(bias) [-> Div(sqrt2) Erf Add(1) Mul(x) Mul(0.5)]
//       => one tensor-core GEMM with a bias (+ Erf-GELU) epilogue; W is
//          re-laid out once as [N, K] (K-major) for the GEMM's TMA loads
//   three such GEMMs on the same input feeding an attention block
//       => one GEMM with concatenated [3N, K] weights
//   Reshape/Transpose -> MatMul(Q, K^T) -> Div(scale) -> Add(mask) ->
//   Softmax -> MatMul(P, V) -> Transpose -> Reshape
//       => one fused attention kernel reading Q/K/V in place
//   [Add(a, b) ->] ReduceMean -> Sub -> Pow(2) -> ReduceMean -> Add(eps) ->
//   Sqrt -> Div -> Mul(gamma) -> Add(beta)
//       => one LayerNorm kernel (with the residual Add folded in)
//   Conv(+Add bias)(+Relu) -> MaxPool -> ... -> Reshape -> MatMul -> Add(bias)
//   on a batch-1 input whose activations fit in shared memory (mnist-8)
//       => one single-CTA kernel for the whole chain (tiny.cu), bit-identical
//          to the per-step kernels it replaces
// A fused step re-checks its shapes at run time and otherwise executes its
// original nodes.  flags & 2 applies Conv's strides/pads/dilations/group
// attributes; without it Conv sees them as absent, as the reference does
// (it reads INTS attributes as int[] while the loader stores long[],
// Node.cs:137-138 vs NodeUtil.cs:13-14).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "lonnx_internal.cuh"

namespace lonnx {
int transpose_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, const int64_t *shape, int rank,
                     const int64_t *perm, void *y);
int strided_copy_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, int rank, const int64_t *out_dims,
                        const int64_t *in_strides, int64_t in_offset, void *y, const int64_t *out_strides);
}

namespace {

using namespace lonnx;

enum DType { DT_FLOAT = 1, DT_INT32 = 6, DT_INT64 = 7, DT_BOOL = 9 };

int dtype_size(int dt) {
    switch (dt) {
    case DT_FLOAT: return 4;
    case DT_INT32: return 4;
    case DT_INT64: return 8;
    case DT_BOOL: return 1;
    default: return 0;
    }
}

struct OpError : std::runtime_error {
    int code;
    OpError(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string &msg) { throw OpError(code, msg); }
void ck(int rc) {
    if (rc) throw OpError(rc, lonnx_last_error());
}

struct DevBuf {
    lonnx_ctx *ctx;
    void *p = nullptr;
    DevBuf(lonnx_ctx *c, size_t bytes) : ctx(c) { ck(ctx_alloc(c, bytes ? bytes : 1, &p)); }
    ~DevBuf() { ctx_free(ctx, p); }
};

struct Value {
    int dtype = DT_FLOAT;
    std::vector<int64_t> shape;
    std::shared_ptr<DevBuf> buf;     // device storage (may be shared by views)
    const void *ext = nullptr;       // caller-owned device pointer
    std::shared_ptr<std::vector<uint8_t>> host;  // host copy (int64 / small constants)
    // device storage is [N, H, W, C] while `shape` stays the logical
    // [N, C, H, W]: a conv-chain value (mark_nhwc); lookup() hands readers
    // that do not ask for it an NCHW copy
    bool nhwc = false;
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
    size_t bytes() const { return (size_t)numel() * dtype_size(dtype); }
    bool on_dev() const { return buf || ext; }
    const void *dptr() const { return ext ? ext : (buf ? buf->p : nullptr); }
    void *dptr_mut() const { return buf ? buf->p : const_cast<void *>(ext); }
    template <typename T>
    const T *h() const { return reinterpret_cast<const T *>(host->data()); }
};

struct Attr {
    int kind = 0;  // 1 int, 2 ints, 3 float, 4 string, 5 floats, 6 tensor
    int64_t i = 0;
    std::vector<int64_t> ints;
    float f = 0;
    std::vector<float> floats;
    std::string s;
    // kind 6: a TensorProto-valued attribute (Constant's `value`)
    int tdtype = 0;
    std::vector<int64_t> tshape;
    std::vector<uint8_t> tdata;
};

struct NodeDef {
    std::string op;
    std::vector<std::string> in, out;
    std::map<std::string, Attr> attrs;
    bool has(const char *n, int kind) const {
        auto it = attrs.find(n);
        return it != attrs.end() && it->second.kind == kind;
    }
    const Attr *get(const char *n) const {
        auto it = attrs.find(n);
        return it == attrs.end() ? nullptr : &it->second;
    }
};

enum StepKind { S_NODE, S_GEMM, S_LN, S_ATTN, S_CONV, S_TINY };

struct Step {
    StepKind kind = S_NODE;
    std::vector<int> nodes;  // original node indices (fallback / S_NODE)
    // GEMM
    std::string x, y;        // input / output names
    std::shared_ptr<DevBuf> wt;   // [N, K] weight, tf32 high parts
    std::shared_ptr<DevBuf> wlo;  // [N, K] low parts (wt + wlo == W^T exactly)
    std::shared_ptr<DevBuf> bias;
    int N = 0, K = 0, epi = 0;
    int w_tapmajor = 0;  // conv: wt / wlo columns in (ky, kx, c) order (NHWC gather)
    int wtrans = 0;          // GEMM from an ONNX Gemm: weight stored [N, K] (transB = 1)
    float bias_beta = 1.0f;  // GEMM from an ONNX Gemm: the bias is beta * C
    std::vector<std::string> split_outputs;  // QKV: outputs per part (views), part width N/parts
    // LN
    std::string a, b;  // x (and residual) inputs
    std::string gamma, beta;
    float eps = 0;
    // ATTN
    std::string q, k, v, mask;
    int heads = 0, dh = 0;
    float scale = 1;
    bool qkv_packed = false;  // q/k/v are column slices of one [T, 3H] GEMM output
    std::string qkv;
    // TINY: a chain of steps run as one small-network kernel when it fits
    std::vector<Step> sub;
};

}  // namespace

struct lonnx_graph {
    lonnx_ctx *ctx;
    std::vector<NodeDef> nodes;
    std::map<std::string, Value> inits;
    std::map<std::string, Value> inputs;
    std::vector<std::string> outputs;
    std::map<std::string, Value> env;
    std::vector<Step> steps;
    bool prepared = false;
    // CUDA-graph capture of one execution (lonnx_graph_capture / _replay)
    cudaGraphExec_t exec = nullptr;
    std::vector<void *> held;                    // blocks the captured graph uses
    std::map<std::string, Value> captured_outputs;
    bool honor_conv_attrs = false;
    int opset = 13;
    std::set<std::string> nhwc_vals;  // values allowed to be stored NHWC (mark_nhwc)
};

namespace {

// ---------------------------------------------------------------------------
// helpers

Value new_dev(lonnx_graph *g, int dtype, const std::vector<int64_t> &shape);

// An NCHW copy of an NHWC-stored value
Value to_nchw(lonnx_graph *g, const Value &v) {
    Value y = new_dev(g, v.dtype, v.shape);
    const int64_t phys[4] = {v.shape[0], v.shape[2], v.shape[3], v.shape[1]}, perm[4] = {0, 3, 1, 2};
    ck(transpose_launch(g->ctx, v.dptr(), (int)dtype_size(v.dtype), phys, 4, perm, y.dptr_mut()));
    return y;
}

// The value as its readers expect it (NCHW): an NHWC-stored value is
// replaced by its NCHW copy the first time a reader that does not handle
// NHWC asks for it.
const Value &lookup(lonnx_graph *g, const std::string &name) {
    auto it = g->env.find(name);
    if (it != g->env.end()) {
        if (it->second.nhwc) {
            static const bool trace = getenv("LONNX_CONV_TRACE") && getenv("LONNX_CONV_TRACE")[0] == '1';
            if (trace) fprintf(stderr, "[lonnx conv] %s: NHWC -> NCHW for a reader\n", name.c_str());
            it->second = to_nchw(g, it->second);
        }
        return it->second;
    }
    auto ii = g->inputs.find(name);
    if (ii != g->inputs.end()) return ii->second;
    auto in = g->inits.find(name);
    if (in != g->inits.end()) return in->second;
    fail(LONNX_E_BADARG, "The required input parameter " + name + " is missing or null.");
}

// The value as stored, for the readers that handle both layouts (check .nhwc)
const Value &lookup_raw(lonnx_graph *g, const std::string &name) {
    auto it = g->env.find(name);
    if (it != g->env.end()) return it->second;
    return lookup(g, name);
}

bool has_value(lonnx_graph *g, const std::string &name) {
    return g->env.count(name) || g->inputs.count(name) || g->inits.count(name);
}

Value new_dev(lonnx_graph *g, int dtype, const std::vector<int64_t> &shape) {
    Value v;
    v.dtype = dtype;
    v.shape = shape;
    v.buf = std::make_shared<DevBuf>(g->ctx, v.bytes());
    return v;
}

void ensure_dev(lonnx_graph *g, Value &v) {
    if (v.on_dev()) return;
    if (!v.host) fail(LONNX_E_BADARG, "tensor has no data");
    v.buf = std::make_shared<DevBuf>(g->ctx, v.bytes());
    ck(lonnx_memcpy_h2d(g->ctx, v.buf->p, v.host->data(), v.bytes()));
}

void ensure_host(lonnx_graph *g, Value &v) {
    if (v.host) return;
    v.host = std::make_shared<std::vector<uint8_t>>(v.bytes());
    ck(lonnx_memcpy_d2h(g->ctx, v.host->data(), v.dptr(), v.bytes()));
}

int64_t norm_axis(int64_t a, int64_t rank) { return a < 0 ? a + rank : a; }

std::vector<int64_t> ints_of(lonnx_graph *g, const std::string &name) {
    Value v = lookup(g, name);
    ensure_host(g, v);
    std::vector<int64_t> r(v.numel());
    if (v.dtype == DT_INT64) memcpy(r.data(), v.host->data(), r.size() * 8);
    else if (v.dtype == DT_INT32) for (size_t i = 0; i < r.size(); ++i) r[i] = v.h<int32_t>()[i];
    else fail(LONNX_E_BADARG, "expected an integer tensor for " + name);
    return r;
}

bool scalar_value(lonnx_graph *g, const std::string &name, float *out) {
    auto it = g->inits.find(name);
    if (it == g->inits.end() || it->second.dtype != DT_FLOAT || it->second.numel() != 1 || !it->second.host) return false;
    *out = it->second.h<float>()[0];
    return true;
}

std::string shape_str(const std::vector<int64_t> &s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
    return r + "]";
}

// conv/pool geometry: MathOps.GetConv2DOutputInfo (src/Lokad.Onnx.Tensors/MathOps.cs:36-89)
struct PadInfo { int oh, ow, top, left, bottom, right; };
PadInfo conv_output_info(int mode, int H, int W, int sh, int sw, int kh, int kw, int pv) {
    PadInfo p{};
    if (mode == 0) {  // VALID
        p.oh = (int)ceil((H - kh + 1.0) / sh);
        p.ow = (int)ceil((W - kw + 1.0) / sw);
    } else if (mode == 1) {  // SAME_UPPER / SAME_LOWER
        p.oh = (int)ceil(H / (float)sh);
        p.ow = (int)ceil(W / (float)sw);
        const int ph = (p.oh - 1) * sh + kh - H, pw = (p.ow - 1) * sw + kw - W;
        p.top = (int)floor(ph / 2.0f);
        p.bottom = ph - p.top;
        p.left = (int)floor(pw / 2.0f);
        p.right = pw - p.left;
    } else {  // explicit symmetric value
        p.top = p.bottom = p.left = p.right = pv;
        p.oh = (int)floor((H - kh + 2.0f * pv) / sh) + 1;
        p.ow = (int)floor((W - kw + 2.0f * pv) / sw) + 1;
    }
    return p;
}

// auto_pad -> mode (CPUExecutionProvider.cs:253-279): 0 VALID, 1 SAME, 2 VALUE
int pad_mode(const NodeDef &n, std::vector<int64_t> *pads, int *pv) {
    const Attr *ap = n.get("auto_pad");
    if (!ap || ap->kind != 4 || ap->s.empty() || ap->s == "VALID") return 0;
    if (ap->s == "SAME_UPPER" || ap->s == "SAME_LOWER") return 1;
    if (ap->s == "NOTSET") {
        if (!pads) fail(LONNX_E_BADARG, "The required attribute pads is missing or null. When auto_pad is NOTSET pads must be specified");
        for (auto p : *pads)
            if (p != (*pads)[0]) fail(LONNX_E_UNSUPPORTED, "The attribute pads is not supported. Asymmetric padding is not supported.");
        *pv = (int)(*pads)[0];
        return 2;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// per-node execution (Node.ExecuteCPU mirror)

int binop_code(const std::string &op) {
    if (op == "Add") return LONNX_ADD;
    if (op == "Sub") return LONNX_SUB;
    if (op == "Mul") return LONNX_MUL;
    if (op == "Div") return LONNX_DIV;
    return LONNX_POW;
}

template <typename T>
T host_binop(int op, T l, T r) {
    switch (op) {
    case LONNX_ADD: return l + r;
    case LONNX_SUB: return l - r;
    case LONNX_MUL: return l * r;
    case LONNX_DIV: return r ? l / r : 0;
    default: return (T)pow((double)l, (double)r);
    }
}

void exec_binary(lonnx_graph *g, const NodeDef &n) {
    Value a = lookup(g, n.in.at(0)), b = lookup(g, n.in.at(1));
    if (a.dtype != b.dtype) fail(LONNX_E_BADARG, "The input tensor " + n.in[1] + " for parameter B has the wrong type: Input tensors must be of the same type..");
    int64_t os[8];
    int orank = 0;
    if (a.shape.size() > 8 || b.shape.size() > 8) fail(LONNX_E_UNSUPPORTED, "rank > 8");
    if (lonnx_broadcast_shape(a.shape.data(), (int)a.shape.size(), b.shape.data(), (int)b.shape.size(), os, &orank))
        fail(LONNX_E_SHAPE, "The tensors " + n.in[0] + shape_str(a.shape) + " and " + n.in[1] + shape_str(b.shape) +
                                " are not compatible for broadcasting.");
    std::vector<int64_t> oshape(os, os + orank);
    const int op = binop_code(n.op);
    if (a.dtype == DT_FLOAT) {
        ensure_dev(g, a);
        ensure_dev(g, b);
        Value y = new_dev(g, DT_FLOAT, oshape);
        ck(lonnx_binary_f32(g->ctx, op, (const float *)a.dptr(), a.shape.data(), (int)a.shape.size(),
                            (const float *)b.dptr(), b.shape.data(), (int)b.shape.size(), (float *)y.dptr_mut()));
        g->env[n.out.at(0)] = y;
        return;
    }
    if (a.dtype != DT_INT64) fail(LONNX_E_UNSUPPORTED, "The type for input parameter A is not supported for operation " + n.op);
    ensure_host(g, a);
    ensure_host(g, b);
    Value y;
    y.dtype = DT_INT64;
    y.shape = oshape;
    y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
    int64_t *yp = (int64_t *)y.host->data();
    const int64_t n_out = y.numel();
    for (int64_t i = 0; i < n_out; ++i) {
        int64_t rem = i, ia = 0, ib = 0, sa = 1, sb = 1;
        for (int d = orank - 1; d >= 0; --d) {
            const int64_t c = rem % oshape[d];
            rem /= oshape[d];
            const int da = d - (orank - (int)a.shape.size()), db = d - (orank - (int)b.shape.size());
            if (da >= 0) { if (a.shape[da] != 1) ia += c * sa; sa *= a.shape[da]; }
            if (db >= 0) { if (b.shape[db] != 1) ib += c * sb; sb *= b.shape[db]; }
        }
        yp[i] = host_binop<int64_t>(op, a.h<int64_t>()[ia], b.h<int64_t>()[ib]);
    }
    g->env[n.out.at(0)] = y;
}

void exec_unary(lonnx_graph *g, const NodeDef &n, int op) {
    Value x = lookup(g, n.in.at(0));
    if (x.dtype != DT_FLOAT) fail(LONNX_E_UNSUPPORTED, "The type for input parameter X is not supported for operation " + n.op);
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, x.shape);
    ck(lonnx_unary_f32(g->ctx, op, (const float *)x.dptr(), (float *)y.dptr_mut(), x.numel()));
    g->env[n.out.at(0)] = y;
}

void exec_matmul(lonnx_graph *g, const NodeDef &n) {
    Value a = lookup(g, n.in.at(0)), b = lookup(g, n.in.at(1));
    if (a.dtype != DT_FLOAT || b.dtype != DT_FLOAT) fail(LONNX_E_UNSUPPORTED, "MatMul: only float tensors are supported on the device");
    ensure_dev(g, a);
    ensure_dev(g, b);
    const int ar = (int)a.shape.size(), br = (int)b.shape.size();
    std::vector<int64_t> oshape;
    if (ar == 1 && br == 1) oshape = {1};
    else if (ar >= 2 && br >= 2) {
        int64_t lead[8];
        int lr = 0;
        if (lonnx_broadcast_shape(a.shape.data(), ar - 2, b.shape.data(), br - 2, lead, &lr))
            fail(LONNX_E_SHAPE, "The tensor shapes are not compatible for broadcasting.");
        oshape.assign(lead, lead + lr);
        oshape.push_back(a.shape[ar - 2]);
        oshape.push_back(b.shape[br - 1]);
    } else {
        fail(LONNX_E_SHAPE, "The shapes " + shape_str(a.shape) + " and " + shape_str(b.shape) + " are not compatible for broadcasting.");
    }
    Value y = new_dev(g, DT_FLOAT, oshape);
    ck(lonnx_matmul_f32(g->ctx, (const float *)a.dptr(), a.shape.data(), ar, (const float *)b.dptr(), b.shape.data(), br,
                        (float *)y.dptr_mut()));
    g->env[n.out.at(0)] = y;
}

// Conv node, optionally fused: relu = a following Relu, res = the other
// input of a following Add (same shape as the Conv output; the caller
// checks), whi/wlo = the weight split at prepare time.
// Conv geometry from the node's attributes (as the reference's op sees them,
// see the file header) and the input / weight shapes
struct ConvGeom {
    int N, C, H, W, M, kh, kw, sh, sw, pt, pl, pb, pr, dh, dw, group, Ho, Wo;
};
ConvGeom conv_geom(lonnx_graph *g, const NodeDef &n, const std::vector<int64_t> &xs, const std::vector<int64_t> &ws) {
    if (xs.size() != 4) fail(LONNX_E_SHAPE, "The input tensor " + n.in[0] + " for parameter X has shape " + shape_str(xs) + " but is required to have rank 4.");
    if (ws.size() != 4) fail(LONNX_E_SHAPE, "The input tensor " + n.in[1] + " for parameter W has shape " + shape_str(ws) + " but is required to have rank 4.");
    std::vector<int64_t> strides{1, 1}, dil{1, 1}, pads_v;
    std::vector<int64_t> *pads = nullptr;
    int group = 1;
    int kh = (int)ws[2], kw = (int)ws[3];
    if (g->honor_conv_attrs) {
        if (const Attr *a = n.get("strides")) strides = a->ints;
        if (const Attr *a = n.get("dilations")) dil = a->ints;
        if (const Attr *a = n.get("pads")) { pads_v = a->ints; pads = &pads_v; }
        if (const Attr *a = n.get("group")) group = (int)a->i;
        if (const Attr *a = n.get("kernel_shape")) { kh = (int)a->ints[0]; kw = (int)a->ints[1]; }
    }
    int pv = 0;
    int mode = pad_mode(n, pads, &pv);
    if (g->honor_conv_attrs && mode == 0 && pads && !n.get("auto_pad")) {
        // ONNX default auto_pad=NOTSET with explicit pads
        for (auto p : *pads) if (p != (*pads)[0]) fail(LONNX_E_UNSUPPORTED, "Asymmetric padding is not supported.");
        mode = 2;
        pv = (int)(*pads)[0];
    }
    ConvGeom c{};
    c.N = (int)xs[0]; c.C = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
    c.M = (int)ws[0]; c.kh = kh; c.kw = kw; c.group = group;
    c.sh = (int)strides[0]; c.sw = (int)strides[1]; c.dh = (int)dil[0]; c.dw = (int)dil[1];
    const int ekh = dil[0] <= 1 ? kh : kh + (kh - 1) * ((int)dil[0] - 1);
    const int ekw = dil[1] <= 1 ? kw : kw + (kw - 1) * ((int)dil[1] - 1);
    PadInfo p = conv_output_info(mode, c.H, c.W, c.sh, c.sw, ekh, ekw, pv);
    // the reference hands (left, top, right, bottom) to MathOps.Conv2D as
    // (padY, padX, padH, padW), TensorOps.cs:937
    c.pt = p.left; c.pl = p.top; c.pb = p.right; c.pr = p.bottom;
    c.Ho = (c.H + c.pt + c.pb - (c.dh * (kh - 1) + 1)) / c.sh + 1;
    c.Wo = (c.W + c.pl + c.pr - (c.dw * (kw - 1) + 1)) / c.sw + 1;
    if (c.Ho != p.oh || c.Wo != p.ow) fail(LONNX_E_SHAPE, "Conv: output geometry mismatch");
    return c;
}

// Conv node, optionally fused: relu = a following Relu, res = the other
// input of a following Add (same shape as the Conv output; the caller
// checks), whi/wlo = the weight split at prepare time.
bool exec_conv(lonnx_graph *g, const NodeDef &n, int relu = 0, const std::string *out_name = nullptr,
               const Value *res = nullptr, const float *whi = nullptr, const float *wlo = nullptr,
               int w_tapmajor = 0, const Value *bias_add = nullptr) {
    Value x = lookup_raw(g, n.in.at(0)), w = lookup(g, n.in.at(1));
    Value bias;
    // bias_add: a following per-channel Add folded in as the bias (the conv
    // has none); the bias pass after the sum is the Add node's one rounding
    const bool has_bias = bias_add || (n.in.size() > 2 && !n.in[2].empty());
    if (bias_add) bias = *bias_add;
    else if (has_bias) bias = lookup(g, n.in[2]);
    if (w.dtype != x.dtype) fail(LONNX_E_BADARG, "The weights tensor must be the same type as the input tensor.");
    const ConvGeom c = conv_geom(g, n, x.shape, w.shape);
    ensure_dev(g, x);
    ensure_dev(g, w);
    if (has_bias) ensure_dev(g, bias);
    Value y = new_dev(g, DT_FLOAT, {c.N, c.M, c.Ho, c.Wo});
    if (res && res->shape != y.shape) return false;
    const std::string &oname = out_name ? *out_name : n.out.at(0);
    int out_nhwc = g->nhwc_vals.count(oname) ? 1 : 0;  // asked for; conv2d says what it wrote
    ck(lonnx::conv2d(g->ctx, (const float *)x.dptr(), (const float *)w.dptr(), whi, wlo,
                     has_bias ? (const float *)bias.dptr() : nullptr, res ? (const float *)res->dptr() : nullptr,
                     (float *)y.dptr_mut(), c.N, c.C, c.H, c.W, c.M, c.kh, c.kw, c.sh, c.sw, c.pt, c.pl, c.pb, c.pr,
                     c.dh, c.dw, c.group, relu, w_tapmajor, x.nhwc ? 1 : 0, res && res->nhwc ? 1 : 0, &out_nhwc));
    y.nhwc = out_nhwc != 0;
    g->env[oname] = y;
    return true;
}

// MaxPool geometry: kernel, strides, pads (top, left) and the output size
struct PoolGeom {
    int N, C, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo;
};
PoolGeom pool_geom(const NodeDef &n, const std::vector<int64_t> &xs) {
    if (xs.size() != 4) fail(LONNX_E_SHAPE, "The input tensor " + n.in[0] + " for parameter X has shape " + shape_str(xs) + " but is required to have rank 4.");
    const Attr *ks = n.get("kernel_shape");
    if (!ks) fail(LONNX_E_BADARG, "kernelshape");
    std::vector<int64_t> strides = ks->ints, dil{1, 1}, pads_v;
    std::vector<int64_t> *pads = nullptr;
    if (const Attr *a = n.get("strides")) strides = a->ints;
    if (const Attr *a = n.get("dilations")) dil = a->ints;
    if (const Attr *a = n.get("pads")) { pads_v = a->ints; pads = &pads_v; }
    int pv = 0;
    const int mode = pad_mode(n, pads, &pv);
    PoolGeom q{};
    q.N = (int)xs[0]; q.C = (int)xs[1]; q.H = (int)xs[2]; q.W = (int)xs[3];
    q.kh = (int)ks->ints[0]; q.kw = (int)ks->ints[1];
    q.sh = (int)strides[0]; q.sw = (int)strides[1];
    const int ekh = dil[0] <= 1 ? q.kh : q.kh + (q.kh - 1) * ((int)dil[0] - 1);
    const int ekw = dil[1] <= 1 ? q.kw : q.kw + (q.kw - 1) * ((int)dil[1] - 1);
    PadInfo p = conv_output_info(mode, q.H, q.W, q.sh, q.sw, ekh, ekw, pv);
    q.pt = p.top; q.pl = p.left; q.Ho = p.oh; q.Wo = p.ow;
    return q;
}

void exec_maxpool(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup_raw(g, n.in.at(0));
    if (x.nhwc && !g->nhwc_vals.count(n.out.at(0))) x = lookup(g, n.in.at(0));
    const PoolGeom q = pool_geom(n, x.shape);
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, {q.N, q.C, q.Ho, q.Wo});
    if (x.nhwc) {  // NHWC in, NHWC out
        ck(lonnx::maxpool2d_nhwc(g->ctx, (const float *)x.dptr(), (float *)y.dptr_mut(), q.N, q.C, q.H, q.W, q.kh,
                                 q.kw, q.sh, q.sw, q.pt, q.pl, q.Ho, q.Wo));
        y.nhwc = true;
        g->env[n.out.at(0)] = y;
        return;
    }
    ck(lonnx_maxpool2d_f32(g->ctx, (const float *)x.dptr(), (float *)y.dptr_mut(), q.N, q.C, q.H, q.W, q.kh, q.kw, q.sh,
                           q.sw, q.pt, q.pl, q.Ho, q.Wo));
    g->env[n.out.at(0)] = y;
}

std::vector<int64_t> reduce_axes(lonnx_graph *g, const NodeDef &n, bool axes_from_attr) {
    if (axes_from_attr) {
        const Attr *a = n.get("axes");
        return a ? a->ints : std::vector<int64_t>{};
    }
    if (n.in.size() > 1 && !n.in[1].empty()) return ints_of(g, n.in[1]);
    if (const Attr *a = n.get("axes")) return a->ints;
    return {};
}

void exec_reduce(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup_raw(g, n.in.at(0));
    if (x.dtype != DT_FLOAT) fail(LONNX_E_UNSUPPORTED, "The operation " + n.op + " is not supported by the backend.");
    const bool attr_axes = (n.op == "ReduceMean" && g->opset < 13);
    std::vector<int64_t> axes = reduce_axes(g, n, attr_axes);
    const int rank = (int)x.shape.size();
    int64_t keep = 1;
    if (const Attr *a = n.get("keepdims")) keep = a->i;
    std::vector<bool> red(rank, axes.empty());
    for (auto a : axes) red[norm_axis(a, rank)] = true;
    std::vector<int64_t> oshape;
    for (int d = 0; d < rank; ++d)
        if (!red[d]) oshape.push_back(x.shape[d]);
        else if (keep) oshape.push_back(1);
    const int op = n.op == "ReduceSum" ? LONNX_REDUCE_SUM : n.op == "ReduceMax" ? LONNX_REDUCE_MAX : LONNX_REDUCE_MEAN;
    if (x.nhwc) {
        if (rank == 4 && !red[0] && !red[1] && red[2] && red[3]) {
            // over H x W of an NHWC value: [N, H*W, C] -> [N, C], the same
            // bits as the NCHW reduction (k_reduce_hw_nhwc)
            Value y = new_dev(g, DT_FLOAT, oshape);
            ck(lonnx::reduce_hw_nhwc(g->ctx, op, (const float *)x.dptr(), (float *)y.dptr_mut(), (int)x.shape[0],
                                     (int)(x.shape[2] * x.shape[3]), (int)x.shape[1]));
            g->env[n.out.at(0)] = y;
            return;
        }
        x = lookup(g, n.in.at(0));
    }
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, oshape);
    ck(lonnx_reduce_f32(g->ctx, op, (const float *)x.dptr(), x.shape.data(), rank, axes.data(), (int)axes.size(),
                        (float *)y.dptr_mut()));
    g->env[n.out.at(0)] = y;
}

void exec_softmax(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const int rank = (int)x.shape.size();
    int64_t axis = -1;
    if (const Attr *a = n.get("axis")) axis = a->i;
    axis = norm_axis(axis, rank);
    if (axis >= rank || axis < 0) fail(LONNX_E_BADARG, "The specified axis must be less than the rank of the tensor.");
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < axis; ++d) outer *= x.shape[d];
    for (int d = (int)axis + 1; d < rank; ++d) inner *= x.shape[d];
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, x.shape);
    ck(lonnx_softmax_f32(g->ctx, (const float *)x.dptr(), (float *)y.dptr_mut(), outer, x.shape[axis], inner));
    g->env[n.out.at(0)] = y;
}

void exec_gather(lonnx_graph *g, const NodeDef &n) {
    Value data = lookup(g, n.in.at(0)), idx = lookup(g, n.in.at(1));
    if (idx.shape.size() > data.shape.size()) fail(LONNX_E_SHAPE, "Gather: indices rank exceeds data rank");
    if (data.shape.empty()) fail(LONNX_E_BADARG, "Cannot gather from a tensor of rank 0.");
    int64_t axis = 0;
    if (const Attr *a = n.get("axis")) axis = a->i;
    const int rank = (int)data.shape.size();
    axis = norm_axis(axis, rank);
    std::vector<int64_t> oshape(data.shape.begin(), data.shape.begin() + axis);
    oshape.insert(oshape.end(), idx.shape.begin(), idx.shape.end());
    oshape.insert(oshape.end(), data.shape.begin() + axis + 1, data.shape.end());
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < axis; ++d) outer *= data.shape[d];
    for (int d = (int)axis + 1; d < rank; ++d) inner *= data.shape[d];
    const int64_t dim = data.shape[axis];
    if (idx.dtype != DT_INT64 && idx.dtype != DT_INT32) fail(LONNX_E_BADARG, "Gather: indices must be integers");
    if (data.dtype == DT_FLOAT || !data.host) {
        ensure_dev(g, data);
        Value idx64 = idx;
        if (idx.dtype == DT_INT32) {
            ensure_host(g, idx);
            idx64 = Value();
            idx64.dtype = DT_INT64;
            idx64.shape = idx.shape;
            idx64.host = std::make_shared<std::vector<uint8_t>>(idx.numel() * 8);
            for (int64_t i = 0; i < idx.numel(); ++i) ((int64_t *)idx64.host->data())[i] = idx.h<int32_t>()[i];
        }
        ensure_dev(g, idx64);
        Value y = new_dev(g, data.dtype, oshape);
        ck(lonnx_gather(g->ctx, data.dptr(), dtype_size(data.dtype), outer, dim, inner, (const int64_t *)idx64.dptr(),
                        idx64.numel(), y.dptr_mut()));
        g->env[n.out.at(0)] = y;
        return;
    }
    // host gather of small integer tensors (shape arithmetic)
    ensure_host(g, data);
    std::vector<int64_t> ii = ints_of(g, n.in[1]);
    const int es = dtype_size(data.dtype);
    Value y;
    y.dtype = data.dtype;
    y.shape = oshape;
    y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
    for (int64_t o = 0; o < outer; ++o)
        for (size_t j = 0; j < ii.size(); ++j) {
            int64_t k = ii[j] < 0 ? ii[j] + dim : ii[j];
            if (k < 0 || k >= dim) fail(LONNX_E_OOB, "Index was outside the bounds of the array.");
            memcpy(y.host->data() + ((o * ii.size() + j) * inner) * es, data.host->data() + ((o * dim + k) * inner) * es,
                   inner * es);
        }
    g->env[n.out.at(0)] = y;
}

void exec_transpose(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const int rank = (int)x.shape.size();
    std::vector<int64_t> perm;
    if (const Attr *a = n.get("perm")) perm = a->ints;
    else for (int d = rank - 1; d >= 0; --d) perm.push_back(d);
    if ((int)perm.size() != rank) fail(LONNX_E_BADARG, "The size of the permutation array must be the rank of the tensor.");
    if (rank <= 1) { g->env[n.out.at(0)] = x; return; }
    std::vector<int64_t> oshape(rank);
    for (int d = 0; d < rank; ++d) oshape[d] = x.shape[norm_axis(perm[d], rank)];
    if (x.on_dev()) {
        Value y = new_dev(g, x.dtype, oshape);
        ck(lonnx_transpose(g->ctx, x.dptr(), dtype_size(x.dtype), x.shape.data(), rank, perm.data(), y.dptr_mut()));
        g->env[n.out.at(0)] = y;
        return;
    }
    ensure_host(g, x);
    Value y;
    y.dtype = x.dtype;
    y.shape = oshape;
    y.host = std::make_shared<std::vector<uint8_t>>(x.bytes());
    const int es = dtype_size(x.dtype);
    std::vector<int64_t> is(rank);
    int64_t s = 1;
    for (int d = rank - 1; d >= 0; --d) { is[d] = s; s *= x.shape[d]; }
    for (int64_t i = 0; i < x.numel(); ++i) {
        int64_t rem = i, off = 0;
        for (int d = rank - 1; d >= 0; --d) { off += (rem % oshape[d]) * is[norm_axis(perm[d], rank)]; rem /= oshape[d]; }
        memcpy(y.host->data() + i * es, x.host->data() + off * es, es);
    }
    g->env[n.out.at(0)] = y;
}

// Reshape's output shape for an input of shape xs (0 copies a dimension
// unless allowzero, one -1 is inferred)
std::vector<int64_t> reshape_shape(lonnx_graph *g, const NodeDef &n, const std::vector<int64_t> &xs) {
    std::vector<int64_t> shp = ints_of(g, n.in.at(1));
    const bool allow_zero = n.get("allowzero") && n.get("allowzero")->i;
    int64_t numel = 1;
    for (auto d : xs) numel *= d;
    int unknown = -1;
    int64_t known = 1;
    std::vector<int64_t> out;
    for (size_t i = 0; i < shp.size(); ++i) {
        if (shp[i] < -1) fail(LONNX_E_BADARG, "A shape dimension cannot be < -1");
        if (shp[i] == -1) {
            if (unknown >= 0) fail(LONNX_E_BADARG, "At most 1 shape dimension can be -1.");
            unknown = (int)i;
            out.push_back(-1);
        } else if (shp[i] == 0 && !allow_zero) {
            out.push_back(xs.at(i));
            known *= xs[i];
        } else {
            out.push_back(shp[i]);
            known *= shp[i];
        }
    }
    if (unknown >= 0) out[unknown] = known ? numel / known : 0;
    int64_t tot = 1;
    for (auto d : out) tot *= d;
    if (tot != numel)
        fail(LONNX_E_SHAPE, "The input tensor cannot be reshaped to the requested shape. Input shape:" + shape_str(xs) +
                                ", requested shape:" + shape_str(out));
    return out;
}

void exec_reshape(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    Value y = x;  // zero-copy view
    y.shape = reshape_shape(g, n, x.shape);
    g->env[n.out.at(0)] = y;
}

void exec_unsqueeze(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    std::vector<int64_t> axes;
    if (g->opset >= 13 && n.in.size() > 1) axes = ints_of(g, n.in[1]);
    else if (const Attr *a = n.get("axes")) axes = a->ints;
    else fail(LONNX_E_BADARG, "The Ints attribute axes is required but was not found.");
    const int r = (int)(x.shape.size() + axes.size());
    std::vector<bool> ins(r, false);
    for (auto a : axes) ins[norm_axis(a, r)] = true;
    std::vector<int64_t> out;
    size_t j = 0;
    for (int d = 0; d < r; ++d) out.push_back(ins[d] ? 1 : x.shape[j++]);
    Value y = x;
    y.shape = out;
    g->env[n.out.at(0)] = y;
}

void exec_cast(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const Attr *to = n.get("to");
    if (!to) fail(LONNX_E_BADARG, "The Int attribute to is required but was not found.");
    const int dt = (int)to->i;
    if (dt == x.dtype) { g->env[n.out.at(0)] = x; return; }
    if (dt == DT_FLOAT && x.dtype == DT_INT64 && x.on_dev()) {
        Value y = new_dev(g, DT_FLOAT, x.shape);
        ck(lonnx_cast_i64_f32(g->ctx, (const int64_t *)x.dptr(), (float *)y.dptr_mut(), x.numel()));
        g->env[n.out.at(0)] = y;
        return;
    }
    ensure_host(g, x);
    Value y;
    y.dtype = dt;
    y.shape = x.shape;
    y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
    for (int64_t i = 0; i < x.numel(); ++i) {
        double v = 0;
        switch (x.dtype) {
        case DT_FLOAT: v = x.h<float>()[i]; break;
        case DT_INT64: v = (double)x.h<int64_t>()[i]; break;
        case DT_INT32: v = x.h<int32_t>()[i]; break;
        case DT_BOOL: v = x.h<uint8_t>()[i]; break;
        default: fail(LONNX_E_UNSUPPORTED, "Cast: source type");
        }
        switch (dt) {
        case DT_FLOAT: ((float *)y.host->data())[i] = (float)v; break;
        case DT_INT64: ((int64_t *)y.host->data())[i] = (int64_t)v; break;
        case DT_INT32: ((int32_t *)y.host->data())[i] = (int32_t)v; break;
        case DT_BOOL: ((uint8_t *)y.host->data())[i] = v != 0; break;
        default: fail(LONNX_E_UNSUPPORTED, "The attribute to is not supported for operation Cast.");
        }
    }
    if (dt == DT_FLOAT) ensure_dev(g, y);
    g->env[n.out.at(0)] = y;
}

void exec_shape(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const int64_t r = (int64_t)x.shape.size();
    int64_t s = 0, e = r;
    if (const Attr *a = n.get("start")) s = a->i;
    if (const Attr *a = n.get("end")) e = a->i;
    s = std::min(std::max(norm_axis(s, r), (int64_t)0), r);
    e = std::min(std::max(norm_axis(e, r), (int64_t)0), r);
    Value y;
    y.dtype = DT_INT64;
    y.shape = {std::max<int64_t>(e - s, 0)};
    y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
    for (int64_t i = s; i < e; ++i) ((int64_t *)y.host->data())[i - s] = x.shape[i];
    g->env[n.out.at(0)] = y;
}

void exec_constant(lonnx_graph *g, const NodeDef &n) {
    Value y;
    if (const Attr *a = n.get("value"); a && a->kind == 6) {
        y.dtype = a->tdtype;
        y.shape = a->tshape;
        y.host = std::make_shared<std::vector<uint8_t>>(a->tdata);
        if (y.host->size() != y.bytes()) fail(LONNX_E_BADARG, "Constant: value tensor size mismatch");
        if (y.dtype == DT_FLOAT) ensure_dev(g, y);
    } else if (const Attr *a = n.get("value_floats")) {
        y.dtype = DT_FLOAT;
        y.shape = {(int64_t)a->floats.size()};
        y.host = std::make_shared<std::vector<uint8_t>>(a->floats.size() * 4);
        if (!a->floats.empty()) memcpy(y.host->data(), a->floats.data(), a->floats.size() * 4);
        ensure_dev(g, y);
    } else if (const Attr *a = n.get("value_float")) {
        y.dtype = DT_FLOAT;
        y.host = std::make_shared<std::vector<uint8_t>>(4);
        memcpy(y.host->data(), &a->f, 4);
        ensure_dev(g, y);
    } else if (const Attr *a = n.get("value_int")) {
        y.dtype = DT_INT64;
        y.host = std::make_shared<std::vector<uint8_t>>(8);
        memcpy(y.host->data(), &a->i, 8);
    } else if (const Attr *a = n.get("value_ints")) {
        y.dtype = DT_INT64;
        y.shape = {(int64_t)a->ints.size()};
        y.host = std::make_shared<std::vector<uint8_t>>(a->ints.size() * 8);
        memcpy(y.host->data(), a->ints.data(), a->ints.size() * 8);
    } else {
        fail(LONNX_E_BADARG, "The required attribute value is missing or null.");
    }
    g->env[n.out.at(0)] = y;
}

// Concat / Slice go through a strided copy on the device (float) or memcpy on the host
void exec_concat(lonnx_graph *g, const NodeDef &n) {
    const Attr *ax = n.get("axis");
    if (!ax) fail(LONNX_E_BADARG, "The Int attribute axis is required but was not found.");
    std::vector<Value> xs;
    for (auto &nm : n.in) xs.push_back(lookup(g, nm));
    const int rank = (int)xs[0].shape.size();
    const int64_t axis = norm_axis(ax->i, rank);
    std::vector<int64_t> oshape = xs[0].shape;
    oshape[axis] = 0;
    for (auto &x : xs) {
        if (x.dtype != xs[0].dtype) fail(LONNX_E_BADARG, "All tensors in a concat operation must have the same type.");
        oshape[axis] += x.shape[axis];
    }
    const bool dev = xs[0].dtype == DT_FLOAT || std::any_of(xs.begin(), xs.end(), [](const Value &v) { return v.on_dev() && !v.host; });
    const int es = dtype_size(xs[0].dtype);
    int64_t outer = 1, inner_out = 1;
    for (int d = 0; d < axis; ++d) outer *= oshape[d];
    for (int d = (int)axis; d < rank; ++d) inner_out *= oshape[d];
    Value y;
    y.dtype = xs[0].dtype;
    y.shape = oshape;
    if (dev) {
        y = new_dev(g, y.dtype, oshape);
        int64_t off = 0;
        for (auto &x : xs) {
            ensure_dev(g, x);
            const int64_t inner = x.numel() / std::max<int64_t>(outer, 1);
            if (inner)
                ck(cudaMemcpy2DAsync((uint8_t *)y.dptr_mut() + off * es, inner_out * es, x.dptr(), inner * es, inner * es,
                                     outer, cudaMemcpyDeviceToDevice, g->ctx->stream) == cudaSuccess ? 0 : LONNX_E_CUDA);
            off += inner;
        }
    } else {
        y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
        int64_t off = 0;
        for (auto &x : xs) {
            ensure_host(g, x);
            const int64_t inner = x.numel() / std::max<int64_t>(outer, 1);
            for (int64_t o = 0; o < outer; ++o)
                memcpy(y.host->data() + (o * inner_out + off) * es, x.host->data() + o * inner * es, inner * es);
            off += inner;
        }
    }
    g->env[n.out.at(0)] = y;
}

void exec_slice(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const int rank = (int)x.shape.size();
    std::vector<int64_t> starts = ints_of(g, n.in.at(1)), ends = ints_of(g, n.in.at(2));
    std::vector<int64_t> axes, steps;
    if (n.in.size() > 3 && !n.in[3].empty()) axes = ints_of(g, n.in[3]);
    else for (size_t i = 0; i < starts.size(); ++i) axes.push_back((int64_t)i);
    if (n.in.size() > 4 && !n.in[4].empty()) steps = ints_of(g, n.in[4]);
    else steps.assign(starts.size(), 1);
    std::vector<int64_t> st(rank, 0), sp(rank, 1), od = x.shape;
    for (size_t i = 0; i < starts.size(); ++i) {
        const int64_t a = norm_axis(axes[i], rank), dim = x.shape[a], step = steps[i];
        if (step == 0) fail(LONNX_E_BADARG, "Slice: step cannot be 0");
        int64_t s = starts[i] < 0 ? starts[i] + dim : starts[i];
        int64_t e = ends[i] < 0 ? ends[i] + dim : ends[i];
        if (step > 0) { s = std::min(std::max(s, (int64_t)0), dim); e = std::min(std::max(e, (int64_t)0), dim); }
        else { s = std::min(std::max(s, (int64_t)-1), dim - 1); e = std::min(std::max(e, (int64_t)-1), dim - 1); }
        st[a] = s;
        sp[a] = step;
        od[a] = step > 0 ? std::max<int64_t>(0, (e - s + step - 1) / step) : std::max<int64_t>(0, (s - e + (-step) - 1) / (-step));
    }
    std::vector<int64_t> is(rank), istr(rank), ostr(rank);
    int64_t s = 1, off = 0;
    for (int d = rank - 1; d >= 0; --d) { is[d] = s; s *= x.shape[d]; }
    for (int d = 0; d < rank; ++d) { istr[d] = is[d] * sp[d]; off += st[d] * is[d]; }
    s = 1;
    for (int d = rank - 1; d >= 0; --d) { ostr[d] = s; s *= od[d]; }
    const int es = dtype_size(x.dtype);
    if (x.on_dev() && !(x.host && x.dtype != DT_FLOAT)) {
        Value y = new_dev(g, x.dtype, od);
        if (y.numel()) ck(strided_copy_launch(g->ctx, x.dptr(), es, rank, od.data(), istr.data(), off, y.dptr_mut(), ostr.data()));
        g->env[n.out.at(0)] = y;
        return;
    }
    ensure_host(g, x);
    Value y;
    y.dtype = x.dtype;
    y.shape = od;
    y.host = std::make_shared<std::vector<uint8_t>>(y.bytes());
    for (int64_t i = 0; i < y.numel(); ++i) {
        int64_t rem = i, o = off;
        for (int d = rank - 1; d >= 0; --d) { o += (rem % od[d]) * istr[d]; rem /= od[d]; }
        memcpy(y.host->data() + i * es, x.host->data() + o * es, es);
    }
    g->env[n.out.at(0)] = y;
}

// ---------------------------------------------------------------------------
// ONNX ops the reference names (OpType.cs) but does not dispatch
// (CPUExecutionProvider.cs:24-50): Gemm, BatchNormalization,
// GlobalAveragePool, Flatten, plus the inference no-ops Identity and
// Dropout.  Semantics follow the ONNX operator specification.

float attr_float(const NodeDef &n, const char *name, float d) {
    const Attr *a = n.get(name);
    if (!a) return d;
    return a->kind == 3 ? a->f : (float)a->i;
}

int64_t attr_int(const NodeDef &n, const char *name, int64_t d) {
    const Attr *a = n.get(name);
    return a && a->kind == 1 ? a->i : d;
}

Value device_scalar(lonnx_graph *g, float v) {
    Value s;
    s.dtype = DT_FLOAT;
    s.host = std::make_shared<std::vector<uint8_t>>(4);
    memcpy(s.host->data(), &v, 4);
    ensure_dev(g, s);
    return s;
}

// Y = alpha * op(A) . op(B) + beta * C, C unidirectionally broadcast to [M, N]
void exec_gemm(lonnx_graph *g, const NodeDef &n) {
    Value a = lookup(g, n.in.at(0)), b = lookup(g, n.in.at(1));
    if (a.dtype != DT_FLOAT || b.dtype != DT_FLOAT) fail(LONNX_E_UNSUPPORTED, "Gemm: only float tensors are supported on the device");
    if (a.shape.size() != 2) fail(LONNX_E_SHAPE, "The input tensor " + n.in[0] + " for parameter A has shape " + shape_str(a.shape) + " but is required to have rank 2.");
    if (b.shape.size() != 2) fail(LONNX_E_SHAPE, "The input tensor " + n.in[1] + " for parameter B has shape " + shape_str(b.shape) + " but is required to have rank 2.");
    const float alpha = attr_float(n, "alpha", 1.0f), beta = attr_float(n, "beta", 1.0f);
    const bool ta = attr_int(n, "transA", 0) != 0, tb = attr_int(n, "transB", 0) != 0;
    const int64_t M = ta ? a.shape[1] : a.shape[0], K = ta ? a.shape[0] : a.shape[1];
    const int64_t Kb = tb ? b.shape[1] : b.shape[0], N = tb ? b.shape[0] : b.shape[1];
    if (K != Kb) fail(LONNX_E_SHAPE, "Gemm: inner dimensions " + shape_str(a.shape) + " and " + shape_str(b.shape) + " do not match.");
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) fail(LONNX_E_UNSUPPORTED, "Gemm: dimension too large");
    ensure_dev(g, a);
    ensure_dev(g, b);
    const float *A = (const float *)a.dptr();
    Value at;
    if (ta) {
        at = new_dev(g, DT_FLOAT, {M, K});
        const int64_t perm[2] = {1, 0};
        ck(lonnx_transpose(g->ctx, a.dptr(), 4, a.shape.data(), 2, perm, at.dptr_mut()));
        A = (const float *)at.dptr();
    }
    const bool has_c = n.in.size() > 2 && !n.in[2].empty();
    Value c;
    bool row_bias = false;
    if (has_c) {
        c = lookup(g, n.in[2]);
        if (c.dtype != DT_FLOAT) fail(LONNX_E_BADARG, "Gemm: C must be a float tensor");
        ensure_dev(g, c);
        row_bias = c.numel() == N && (c.shape.size() == 1 || (c.shape.size() == 2 && c.shape[0] == 1));
        int64_t os[8];
        int orank = 0;
        const int64_t mn[2] = {M, N};
        if (c.shape.size() > 2 || lonnx_broadcast_shape(c.shape.data(), (int)c.shape.size(), mn, 2, os, &orank) ||
            orank != 2 || os[0] != M || os[1] != N)
            fail(LONNX_E_SHAPE, "Gemm: C of shape " + shape_str(c.shape) + " does not broadcast to " + shape_str({M, N}));
    }
    Value y = new_dev(g, DT_FLOAT, {M, N});
    ck(lonnx_gemm_f32(g->ctx, A, (const float *)b.dptr(), row_bias ? (const float *)c.dptr() : nullptr,
                      (float *)y.dptr_mut(), 1, (int)M, (int)N, (int)K, 0, 0, 0, tb ? 1 : 0, alpha,
                      row_bias ? beta : 0.0f, LONNX_EPI_NONE));
    if (has_c && !row_bias && beta != 0.0f) {
        Value cb = c;
        if (beta != 1.0f) {
            Value bs = device_scalar(g, beta);
            cb = new_dev(g, DT_FLOAT, c.shape);
            ck(lonnx_binary_f32(g->ctx, LONNX_MUL, (const float *)c.dptr(), c.shape.data(), (int)c.shape.size(),
                                (const float *)bs.dptr(), nullptr, 0, (float *)cb.dptr_mut()));
        }
        Value y2 = new_dev(g, DT_FLOAT, {M, N});
        ck(lonnx_binary_f32(g->ctx, LONNX_ADD, (const float *)y.dptr(), y.shape.data(), 2, (const float *)cb.dptr(),
                            cb.shape.data(), (int)cb.shape.size(), (float *)y2.dptr_mut()));
        y = y2;
    }
    g->env[n.out.at(0)] = y;
}

// mean over every spatial axis (2 .. rank-1), keeping them as 1s
void exec_global_avg_pool(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    if (x.dtype != DT_FLOAT) fail(LONNX_E_UNSUPPORTED, "GlobalAveragePool: only float tensors are supported");
    const int rank = (int)x.shape.size();
    if (rank < 3) fail(LONNX_E_SHAPE, "The input tensor " + n.in[0] + " for parameter X has shape " + shape_str(x.shape) + " but is required to have rank >= 3.");
    std::vector<int64_t> axes, oshape(x.shape.begin(), x.shape.begin() + 2);
    for (int d = 2; d < rank; ++d) { axes.push_back(d); oshape.push_back(1); }
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, oshape);
    ck(lonnx_reduce_f32(g->ctx, LONNX_REDUCE_MEAN, (const float *)x.dptr(), x.shape.data(), rank, axes.data(),
                        (int)axes.size(), (float *)y.dptr_mut()));
    g->env[n.out.at(0)] = y;
}

void exec_flatten(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    const int64_t rank = (int64_t)x.shape.size();
    int64_t axis = norm_axis(attr_int(n, "axis", 1), rank);
    if (axis < 0 || axis > rank) fail(LONNX_E_BADARG, "Flatten: axis out of range");
    int64_t outer = 1;
    for (int64_t d = 0; d < axis; ++d) outer *= x.shape[d];
    Value y = x;  // zero-copy view
    y.shape = {outer, outer ? x.numel() / outer : 0};
    g->env[n.out.at(0)] = y;
}

// inference-mode BatchNormalization over axis 1
void exec_batchnorm(lonnx_graph *g, const NodeDef &n) {
    if (n.in.size() < 5) fail(LONNX_E_BADARG, "BatchNormalization needs X, scale, B, input_mean and input_var");
    if (attr_int(n, "training_mode", 0)) fail(LONNX_E_UNSUPPORTED, "BatchNormalization: training_mode is not supported");
    Value x = lookup(g, n.in[0]);
    Value p[4] = {lookup(g, n.in[1]), lookup(g, n.in[2]), lookup(g, n.in[3]), lookup(g, n.in[4])};
    if (x.dtype != DT_FLOAT || x.shape.size() < 2) fail(LONNX_E_SHAPE, "BatchNormalization: X must be a float tensor of rank >= 2");
    const int64_t C = x.shape[1];
    for (auto &v : p) {
        if (v.dtype != DT_FLOAT || v.numel() != C) fail(LONNX_E_SHAPE, "BatchNormalization: parameters must hold one float per channel");
        ensure_dev(g, v);
    }
    int64_t inner = 1;
    for (size_t d = 2; d < x.shape.size(); ++d) inner *= x.shape[d];
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, x.shape);
    ck(lonnx_batchnorm_f32(g->ctx, (const float *)x.dptr(), (const float *)p[0].dptr(), (const float *)p[1].dptr(),
                           (const float *)p[2].dptr(), (const float *)p[3].dptr(), attr_float(n, "epsilon", 1e-5f),
                           (float *)y.dptr_mut(), x.shape[0], C, inner));
    g->env[n.out.at(0)] = y;
}

// Identity, and Dropout at inference (output = input, mask = all true)
void exec_identity(lonnx_graph *g, const NodeDef &n) {
    Value x = lookup(g, n.in.at(0));
    g->env[n.out.at(0)] = x;
    if (n.out.size() > 1 && !n.out[1].empty()) {
        Value m;
        m.dtype = DT_BOOL;
        m.shape = x.shape;
        m.host = std::make_shared<std::vector<uint8_t>>(m.bytes(), 1);
        g->env[n.out[1]] = m;
    }
}

void exec_node(lonnx_graph *g, const NodeDef &n) {
    const std::string &op = n.op;
    if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div" || op == "Pow") return exec_binary(g, n);
    if (op == "Relu") return exec_unary(g, n, LONNX_RELU);
    if (op == "Sqrt") return exec_unary(g, n, LONNX_SQRT);
    if (op == "Erf") return exec_unary(g, n, LONNX_ERF);
    if (op == "MatMul") return exec_matmul(g, n);
    if (op == "Conv") { exec_conv(g, n); return; }
    if (op == "MaxPool") return exec_maxpool(g, n);
    if (op == "ReduceMean" || op == "ReduceSum" || op == "ReduceMax") return exec_reduce(g, n);
    if (op == "Softmax") return exec_softmax(g, n);
    if (op == "Gather") return exec_gather(g, n);
    if (op == "Transpose") return exec_transpose(g, n);
    if (op == "Reshape") return exec_reshape(g, n);
    if (op == "Unsqueeze") return exec_unsqueeze(g, n);
    if (op == "Cast") return exec_cast(g, n);
    if (op == "Shape") return exec_shape(g, n);
    if (op == "Constant") return exec_constant(g, n);
    if (op == "Concat") return exec_concat(g, n);
    if (op == "Slice") return exec_slice(g, n);
    if (op == "Gemm") return exec_gemm(g, n);
    if (op == "GlobalAveragePool") return exec_global_avg_pool(g, n);
    if (op == "Flatten") return exec_flatten(g, n);
    if (op == "BatchNormalization") return exec_batchnorm(g, n);
    if (op == "Identity" || op == "Dropout") return exec_identity(g, n);
    fail(LONNX_E_UNSUPPORTED, "The operation " + op + " is not supported by the backend.");
}

// ---------------------------------------------------------------------------
// fused steps

bool exec_gemm_step(lonnx_graph *g, const Step &s) {
    const Value &x = lookup(g, s.x);
    if (x.dtype != DT_FLOAT || x.shape.empty() || x.shape.back() != s.K) return false;
    Value xv = x;
    ensure_dev(g, xv);
    const int64_t M = xv.numel() / s.K;
    std::vector<int64_t> oshape = xv.shape;
    oshape.back() = s.N;
    Value y = new_dev(g, DT_FLOAT, oshape);
    const float *bias = s.bias ? (const float *)s.bias->p : nullptr;
    int rc = LONNX_E_UNSUPPORTED;
    if ((int64_t)M * s.N * s.K >= gemm_tc_min_work() && s.K % 4 == 0)
        rc = gemm_tc(g->ctx, (const float *)xv.dptr(), (const float *)s.wt->p, (const float *)s.wlo->p, bias,
                     (float *)y.dptr_mut(), (int)M, s.N, s.K, s.K, s.K, s.N, 1.0f, 1.0f, s.epi);
    if (rc == LONNX_E_UNSUPPORTED) {
        // exact-order FFMA kernel on W^T = hi + lo (reassembled in scratch)
        void *wfull = nullptr;
        ck(ctx_scratch(g->ctx, (size_t)s.N * s.K * 4, &wfull));
        const int64_t shp[1] = {(int64_t)s.N * s.K};
        ck(lonnx_binary_f32(g->ctx, LONNX_ADD, (const float *)s.wt->p, shp, 1, (const float *)s.wlo->p, shp, 1,
                            (float *)wfull));
        rc = gemm_simt(g->ctx, (const float *)xv.dptr(), (const float *)wfull, bias, (float *)y.dptr_mut(), 1, (int)M,
                       s.N, s.K, 0, 0, 0, 1, 1.0f, 1.0f, s.epi, nullptr);
    }
    ck(rc);
    g->env[s.y] = y;
    return true;
}

bool exec_ln_step(lonnx_graph *g, const Step &s) {
    Value x = lookup(g, s.a);
    const Value *r = s.b.empty() ? nullptr : &lookup(g, s.b);
    if (x.dtype != DT_FLOAT || x.shape.empty()) return false;
    if (r && r->dtype != DT_FLOAT) return false;
    if (r && r->shape != x.shape) {
        // a broadcasting Add (the embedding sum plus [S, H] position
        // embeddings): run that Add on its own, then the LayerNorm on its sum
        int64_t os[8];
        int orank = 0;
        if (x.shape.size() > 8 || r->shape.size() > 8 ||
            lonnx_broadcast_shape(x.shape.data(), (int)x.shape.size(), r->shape.data(), (int)r->shape.size(), os,
                                  &orank))
            return false;
        std::vector<int64_t> bshape(os, os + orank);
        const Value &gm0 = lookup(g, s.gamma), &bt0 = lookup(g, s.beta);
        if (bshape.empty() || gm0.numel() != bshape.back() || bt0.numel() != bshape.back()) return false;
        Value rr = *r;
        ensure_dev(g, x);
        ensure_dev(g, rr);
        Value sum = new_dev(g, DT_FLOAT, bshape);
        ck(lonnx_binary_f32(g->ctx, LONNX_ADD, (const float *)x.dptr(), x.shape.data(), (int)x.shape.size(),
                            (const float *)rr.dptr(), rr.shape.data(), (int)rr.shape.size(), (float *)sum.dptr_mut()));
        x = sum;
        r = nullptr;
    }
    const Value &gm = lookup(g, s.gamma), &bt = lookup(g, s.beta);
    const int64_t cols = x.shape.back();
    if (gm.numel() != cols || bt.numel() != cols) return false;
    Value rv;
    if (r) { rv = *r; ensure_dev(g, rv); }
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, x.shape);
    ck(lonnx_layernorm_f32(g->ctx, (const float *)x.dptr(), r ? (const float *)rv.dptr() : nullptr, (const float *)gm.dptr(),
                           (const float *)bt.dptr(), s.eps, (float *)y.dptr_mut(), x.numel() / cols, (int)cols));
    g->env[s.y] = y;
    return true;
}

bool exec_attn_step(lonnx_graph *g, const Step &s) {
    const int H = s.heads * s.dh;
    const float *qp, *kp, *vp;
    int64_t ld;
    std::vector<int64_t> shp;
    if (s.qkv_packed) {
        const Value &qkv = lookup(g, s.qkv);
        if (qkv.shape.size() != 3 || qkv.shape[2] != 3 * H) return false;
        qp = (const float *)qkv.dptr();
        kp = qp + H;
        vp = qp + 2 * H;
        ld = 3 * H;
        shp = qkv.shape;
    } else {
        const Value &q = lookup(g, s.q), &k = lookup(g, s.k), &v = lookup(g, s.v);
        if (q.shape.size() != 3 || q.shape[2] != H || k.shape != q.shape || v.shape != q.shape) return false;
        qp = (const float *)q.dptr();
        kp = (const float *)k.dptr();
        vp = (const float *)v.dptr();
        ld = H;
        shp = q.shape;
    }
    const int B = (int)shp[0], S = (int)shp[1];
    const Value &m = lookup(g, s.mask);
    if (m.dtype != DT_FLOAT || m.numel() != (int64_t)B * S || m.shape.size() != 4 || m.shape[0] != B || m.shape[3] != S)
        return false;
    Value mv = m;
    ensure_dev(g, mv);
    Value y = new_dev(g, DT_FLOAT, {B, S, H});
    ck(lonnx_attention_f32(g->ctx, qp, kp, vp, ld, (const float *)mv.dptr(), (float *)y.dptr_mut(), B, S, s.heads, s.dh,
                           s.scale));
    g->env[s.y] = y;
    return true;
}

// ---------------------------------------------------------------------------
// fusion pass

struct Matcher {
    lonnx_graph *g;
    std::map<std::string, int> producer;
    std::map<std::string, std::vector<int>> consumers;
    std::set<std::string> graph_outputs;
    std::vector<bool> used;

    explicit Matcher(lonnx_graph *gr) : g(gr), used(gr->nodes.size(), false) {
        for (size_t i = 0; i < g->nodes.size(); ++i) {
            for (auto &o : g->nodes[i].out) producer[o] = (int)i;
            for (auto &in : g->nodes[i].in) consumers[in].push_back((int)i);
        }
        for (auto &o : g->outputs) graph_outputs.insert(o);
    }
    // the single consumer of `name` (and name is not a graph output), or -1
    int only_consumer(const std::string &name) const {
        if (graph_outputs.count(name)) return -1;
        auto it = consumers.find(name);
        if (it == consumers.end() || it->second.size() != 1) return -1;
        return it->second[0];
    }
    const NodeDef &N(int i) const { return g->nodes[i]; }
    bool is_init(const std::string &n) const { return g->inits.count(n) > 0; }
    bool scalar_is(const std::string &n, float v, float tol = 0) const {
        float x;
        if (!scalar_value(g, n, &x)) return false;
        return tol == 0 ? x == v : fabsf(x - v) <= tol * fabsf(v);
    }
    bool free(int i) const { return i >= 0 && !used[i]; }
};

// MatMul(x, W) -> Add(., b) [-> GELU chain]
bool match_gemm(Matcher &m, int i, Step &st) {
    const NodeDef &mm = m.N(i);
    if (mm.op != "MatMul" || mm.in.size() != 2 || !m.is_init(mm.in[1])) return false;
    const Value &W = m.g->inits.at(mm.in[1]);
    if (W.dtype != DT_FLOAT || W.shape.size() != 2) return false;
    const int K = (int)W.shape[0], Nn = (int)W.shape[1];
    int a = m.only_consumer(mm.out[0]);
    if (!m.free(a)) return false;
    const NodeDef &add = m.N(a);
    if (add.op != "Add") return false;
    const std::string bname = add.in[0] == mm.out[0] ? add.in[1] : add.in[0];
    if (!m.is_init(bname)) return false;
    const Value &b = m.g->inits.at(bname);
    if (b.dtype != DT_FLOAT || b.numel() != Nn || b.shape.size() != 1) return false;
    st = Step();
    st.kind = S_GEMM;
    st.nodes = {i, a};
    st.x = mm.in[0];
    st.y = add.out[0];
    st.K = K;
    st.N = Nn;
    st.epi = LONNX_EPI_NONE;
    st.a = mm.in[1];  // weight name (re-laid out later)
    st.b = bname;
    // GELU: Div(y, sqrt2) -> Erf -> Add(., 1) -> Mul(y, .) -> Mul(., 0.5)
    const std::string y = add.out[0];
    auto it = m.consumers.find(y);
    if (m.graph_outputs.count(y) || it == m.consumers.end() || it->second.size() != 2) return true;
    int dv = -1, ml = -1;
    for (int c : it->second) {
        if (m.N(c).op == "Div") dv = c;
        if (m.N(c).op == "Mul") ml = c;
    }
    if (!m.free(dv) || !m.free(ml)) return true;
    const NodeDef &D = m.N(dv);
    if (D.in[0] != y || !m.scalar_is(D.in[1], (float)M_SQRT2, 1e-6f)) return true;
    int e = m.only_consumer(D.out[0]);
    if (!m.free(e) || m.N(e).op != "Erf") return true;
    int p1 = m.only_consumer(m.N(e).out[0]);
    if (!m.free(p1) || m.N(p1).op != "Add") return true;
    const NodeDef &P1 = m.N(p1);
    const std::string one = P1.in[0] == m.N(e).out[0] ? P1.in[1] : P1.in[0];
    if (!m.scalar_is(one, 1.0f)) return true;
    const NodeDef &ML = m.N(ml);
    if (!((ML.in[0] == y && ML.in[1] == P1.out[0]) || (ML.in[1] == y && ML.in[0] == P1.out[0]))) return true;
    if (m.only_consumer(P1.out[0]) != ml) return true;
    int h = m.only_consumer(ML.out[0]);
    if (!m.free(h) || m.N(h).op != "Mul") return true;
    const NodeDef &HH = m.N(h);
    const std::string half = HH.in[0] == ML.out[0] ? HH.in[1] : HH.in[0];
    if (!m.scalar_is(half, 0.5f)) return true;
    st.nodes = {i, a, dv, e, p1, ml, h};
    st.y = HH.out[0];
    st.epi = LONNX_EPI_GELU_ERF;
    return true;
}

// [Add(a, b) ->] ReduceMean -> Sub -> Pow(2) -> ReduceMean -> Add(eps) -> Sqrt -> Div -> Mul(gamma) -> Add(beta)
bool match_ln(Matcher &m, int i, Step &st) {
    const NodeDef &r1 = m.N(i);
    if (r1.op != "ReduceMean") return false;
    auto last_axis = [&](const NodeDef &n) {
        std::vector<int64_t> ax;
        if (n.in.size() > 1 && !n.in[1].empty()) {
            if (!m.is_init(n.in[1])) return false;
            ax = ints_of(m.g, n.in[1]);
        } else if (const Attr *a = n.get("axes")) {
            ax = a->ints;
        }
        const Attr *kd = n.get("keepdims");
        return ax.size() == 1 && ax[0] == -1 && (!kd || kd->i == 1);
    };
    if (!last_axis(r1)) return false;
    const std::string x = r1.in[0];
    auto it = m.consumers.find(x);
    if (it == m.consumers.end() || it->second.size() != 2) return false;
    int sb = -1;
    for (int c : it->second) if (c != i) sb = c;
    if (!m.free(sb) || m.N(sb).op != "Sub" || m.N(sb).in[0] != x || m.N(sb).in[1] != r1.out[0]) return false;
    if (m.only_consumer(r1.out[0]) != sb) return false;
    const std::string d = m.N(sb).out[0];
    auto dc = m.consumers.find(d);
    if (m.graph_outputs.count(d) || dc == m.consumers.end() || dc->second.size() != 2) return false;
    int pw = -1, dv = -1;
    for (int c : dc->second) {
        if (m.N(c).op == "Pow") pw = c;
        if (m.N(c).op == "Div") dv = c;
    }
    if (!m.free(pw) || !m.free(dv)) return false;
    if (m.N(pw).in[0] != d || !m.scalar_is(m.N(pw).in[1], 2.0f) || m.N(dv).in[0] != d) return false;
    int r2 = m.only_consumer(m.N(pw).out[0]);
    if (!m.free(r2) || m.N(r2).op != "ReduceMean" || !last_axis(m.N(r2))) return false;
    int ae = m.only_consumer(m.N(r2).out[0]);
    if (!m.free(ae) || m.N(ae).op != "Add") return false;
    const NodeDef &AE = m.N(ae);
    const std::string epsn = AE.in[0] == m.N(r2).out[0] ? AE.in[1] : AE.in[0];
    float eps;
    if (!scalar_value(m.g, epsn, &eps)) return false;
    int sq = m.only_consumer(AE.out[0]);
    if (!m.free(sq) || m.N(sq).op != "Sqrt") return false;
    if (m.only_consumer(m.N(sq).out[0]) != dv || m.N(dv).in[1] != m.N(sq).out[0]) return false;
    int mg = m.only_consumer(m.N(dv).out[0]);
    if (!m.free(mg) || m.N(mg).op != "Mul") return false;
    const NodeDef &MG = m.N(mg);
    if (MG.in[0] != m.N(dv).out[0] || !m.is_init(MG.in[1])) return false;
    int ab = m.only_consumer(MG.out[0]);
    if (!m.free(ab) || m.N(ab).op != "Add") return false;
    const NodeDef &AB = m.N(ab);
    if (AB.in[0] != MG.out[0] || !m.is_init(AB.in[1])) return false;
    st = Step();
    st.kind = S_LN;
    st.nodes = {i, sb, pw, r2, ae, sq, dv, mg, ab};
    st.a = x;
    st.gamma = MG.in[1];
    st.beta = AB.in[1];
    st.eps = eps;
    st.y = AB.out[0];
    // residual Add producing x, used only by this LayerNorm
    auto pi = m.producer.find(x);
    if (pi != m.producer.end() && m.free(pi->second) && m.N(pi->second).op == "Add" && !m.graph_outputs.count(x)) {
        const NodeDef &R = m.N(pi->second);
        if (!m.is_init(R.in[0]) && !m.is_init(R.in[1])) {
            st.a = R.in[0];
            st.b = R.in[1];
            st.nodes.insert(st.nodes.begin(), pi->second);
        }
    }
    return true;
}

// Reshape/Transpose head split -> QK^T -> /scale -> +mask -> Softmax -> PV -> merge
bool match_attn(Matcher &m, int i, Step &st, std::vector<int> &heads_nodes) {
    const NodeDef &s1 = m.N(i);
    if (s1.op != "MatMul") return false;
    auto split = [&](const std::string &t, const std::vector<int64_t> &perm, std::string *src, int *h, int *dh,
                     std::vector<int> *nodes) {
        auto pt = m.producer.find(t);
        if (pt == m.producer.end() || !m.free(pt->second)) return false;
        const NodeDef &T = m.N(pt->second);
        const Attr *pa = T.get("perm");
        if (T.op != "Transpose" || !pa || pa->ints != perm) return false;
        if (m.only_consumer(T.out[0]) < 0) return false;
        auto pr = m.producer.find(T.in[0]);
        if (pr == m.producer.end() || !m.free(pr->second)) return false;
        const NodeDef &R = m.N(pr->second);
        if (R.op != "Reshape" || m.only_consumer(R.out[0]) != pt->second || !m.is_init(R.in[1])) return false;
        std::vector<int64_t> shp = ints_of(m.g, R.in[1]);
        if (shp.size() != 4 || shp[2] <= 0 || shp[3] <= 0) return false;
        if (m.only_consumer(R.in[0]) != pr->second) return false;
        *src = R.in[0];
        *h = (int)shp[2];
        *dh = (int)shp[3];
        nodes->push_back(pr->second);
        nodes->push_back(pt->second);
        return true;
    };
    std::vector<int> nodes;
    std::string q, k, v;
    int hq, dq, hk, dk, hv, dv;
    if (!split(s1.in[0], {0, 2, 1, 3}, &q, &hq, &dq, &nodes)) return false;
    if (!split(s1.in[1], {0, 2, 3, 1}, &k, &hk, &dk, &nodes)) return false;
    if (hq != hk || dq != dk) return false;
    int dvn = m.only_consumer(s1.out[0]);
    if (!m.free(dvn)) return false;
    const NodeDef &DV = m.N(dvn);
    float scale;
    if (DV.op == "Div" && DV.in[0] == s1.out[0] && scalar_value(m.g, DV.in[1], &scale)) {
    } else return false;
    int am = m.only_consumer(DV.out[0]);
    if (!m.free(am) || m.N(am).op != "Add") return false;
    const NodeDef &AM = m.N(am);
    const std::string mask = AM.in[0] == DV.out[0] ? AM.in[1] : AM.in[0];
    int sm = m.only_consumer(AM.out[0]);
    if (!m.free(sm) || m.N(sm).op != "Softmax") return false;
    const Attr *sa = m.N(sm).get("axis");
    if (sa && sa->i != -1 && sa->i != 3) return false;
    int pv = m.only_consumer(m.N(sm).out[0]);
    if (!m.free(pv) || m.N(pv).op != "MatMul" || m.N(pv).in[0] != m.N(sm).out[0]) return false;
    if (!split(m.N(pv).in[1], {0, 2, 1, 3}, &v, &hv, &dv, &nodes)) return false;
    if (hv != hq || dv != dq) return false;
    int tc = m.only_consumer(m.N(pv).out[0]);
    if (!m.free(tc) || m.N(tc).op != "Transpose") return false;
    const Attr *tp = m.N(tc).get("perm");
    if (!tp || tp->ints != std::vector<int64_t>{0, 2, 1, 3}) return false;
    int rs = m.only_consumer(m.N(tc).out[0]);
    if (!m.free(rs) || m.N(rs).op != "Reshape" || !m.is_init(m.N(rs).in[1])) return false;
    std::vector<int64_t> rsh = ints_of(m.g, m.N(rs).in[1]);
    if (rsh.size() != 3 || !(rsh[2] == hq * dq) || !(rsh[0] == 0 || rsh[0] > 0) || !(rsh[1] == 0 || rsh[1] > 0)) return false;
    st = Step();
    st.kind = S_ATTN;
    heads_nodes = nodes;
    st.nodes = nodes;
    for (int n : {i, dvn, am, sm, pv, tc, rs}) st.nodes.push_back(n);
    std::sort(st.nodes.begin(), st.nodes.end());
    st.q = q;
    st.k = k;
    st.v = v;
    st.mask = mask;
    st.heads = hq;
    st.dh = dq;
    st.scale = scale;
    st.y = m.N(rs).out[0];
    return true;
}

// ONNX Gemm(A, W, C) with W an initializer, transA = 0, alpha = 1 and C
// absent or a row bias [N] / [1, N] initializer: one GEMM step (beta folded
// into the bias, transB into the weight split)
bool match_gemm_onnx(Matcher &m, int i, Step &st) {
    const NodeDef &gm = m.N(i);
    if (gm.op != "Gemm" || gm.in.size() < 2 || !m.is_init(gm.in[1])) return false;
    if (attr_int(gm, "transA", 0) != 0 || attr_float(gm, "alpha", 1.0f) != 1.0f) return false;
    const Value &W = m.g->inits.at(gm.in[1]);
    if (W.dtype != DT_FLOAT || W.shape.size() != 2) return false;
    const int tb = attr_int(gm, "transB", 0) ? 1 : 0;
    const int64_t K = tb ? W.shape[1] : W.shape[0], N = tb ? W.shape[0] : W.shape[1];
    if (K > INT32_MAX || N > INT32_MAX) return false;
    std::string bname;
    if (gm.in.size() > 2 && !gm.in[2].empty()) {
        bname = gm.in[2];
        if (!m.is_init(bname)) return false;
        const Value &b = m.g->inits.at(bname);
        if (b.dtype != DT_FLOAT || b.numel() != N || !(b.shape.size() == 1 || (b.shape.size() == 2 && b.shape[0] == 1)))
            return false;
    }
    st = Step();
    st.kind = S_GEMM;
    st.nodes = {i};
    st.x = gm.in[0];
    st.y = gm.out[0];
    st.K = (int)K;
    st.N = (int)N;
    st.epi = LONNX_EPI_NONE;
    st.a = gm.in[1];
    st.b = bname;
    st.wtrans = tb;
    st.bias_beta = attr_float(gm, "beta", 1.0f);
    return true;
}

// Conv [-> Add(residual)] [-> Relu]: each intermediate used only by the next node
bool match_conv(Matcher &m, int i, Step &st) {
    const NodeDef &c = m.N(i);
    if (c.op != "Conv") return false;
    st = Step();
    st.kind = S_CONV;
    st.nodes = {i};
    st.y = c.out[0];
    int nx = m.only_consumer(c.out[0]);
    if (m.free(nx) && m.N(nx).op == "Add" && m.N(nx).in.size() == 2 && m.N(nx).in[0] != m.N(nx).in[1]) {
        const NodeDef &A = m.N(nx);
        st.b = A.in[0] == c.out[0] ? A.in[1] : A.in[0];
        st.nodes.push_back(nx);
        st.y = A.out[0];
        nx = m.only_consumer(A.out[0]);
    }
    if (m.free(nx) && m.N(nx).op == "Relu") {
        st.epi = 1;
        st.nodes.push_back(nx);
        st.y = m.N(nx).out[0];
    }
    if (st.nodes.size() == 1 && !m.is_init(c.in.size() > 1 ? c.in[1] : std::string())) return false;
    return true;
}

bool channel_bias_shape(const Value &v, int64_t M);

// Fused Conv step; false (nothing run) when the residual's shape differs
// from the Conv output, so the nodes run one by one instead.
bool exec_conv_step(lonnx_graph *g, const Step &s) {
    const NodeDef &c = g->nodes[s.nodes[0]];
    Value res;
    if (!s.b.empty()) {
        res = lookup_raw(g, s.b);
        if (res.dtype != DT_FLOAT) return false;
        Value x = lookup_raw(g, c.in.at(0)), w = lookup(g, c.in.at(1));  // shapes only: no relayout
        const bool conv_bias = c.in.size() > 2 && !c.in[2].empty();
        if (!conv_bias && w.shape.size() == 4 && x.shape.size() == 4 && channel_bias_shape(res, w.shape[0])) {
            ensure_dev(g, res);
            const float *whi = s.wt ? (const float *)s.wt->p : nullptr;
            const float *wlo = s.wlo ? (const float *)s.wlo->p : nullptr;
            return exec_conv(g, c, s.epi, &s.y, nullptr, whi, wlo, s.w_tapmajor, &res);
        }
        if (res.shape.size() != 4 || x.shape.size() != 4 || w.shape.size() != 4 || res.shape[0] != x.shape[0] ||
            res.shape[1] != w.shape[0])
            return false;  // exec_conv checks the full shape once it knows Ho, Wo
        ensure_dev(g, res);
    }
    const float *whi = s.wt ? (const float *)s.wt->p : nullptr, *wlo = s.wlo ? (const float *)s.wlo->p : nullptr;
    return exec_conv(g, c, s.epi, &s.y, s.b.empty() ? nullptr : &res, whi, wlo, s.w_tapmajor);
}

// Conv -> Add(per-channel [.., M, 1, 1] operand) [-> Relu] with no conv bias:
// the Add operand becomes the conv's bias.
bool channel_bias_shape(const Value &v, int64_t M) {
    const size_t r = v.shape.size();
    if (r < 3 || v.shape[r - 1] != 1 || v.shape[r - 2] != 1 || v.shape[r - 3] != M) return false;
    for (size_t d = 0; d + 3 < r; ++d)
        if (v.shape[d] != 1) return false;
    return true;
}

Value make_value(lonnx_graph *g, int dtype, const int64_t *shape, int rank, const void *host, bool upload);

// Conv (initializer weight, optional initializer bias) -> BatchNormalization
// (initializer parameters, the conv output used by nothing else): the BN is
// folded into the conv once, W' = W * s and b' = (b - mean) * s + B with
// s = scale / sqrt(var + eps) (computed in double, rounded once), and the BN
// node is removed.  The conv then fuses with a following Add / Relu as usual.
void fold_batchnorm(lonnx_graph *g) {
    std::map<std::string, int> uses, producer;
    for (size_t j = 0; j < g->nodes.size(); ++j) {
        for (auto &in : g->nodes[j].in) uses[in]++;
        for (auto &o : g->nodes[j].out) producer[o] = (int)j;
    }
    const std::set<std::string> outs(g->outputs.begin(), g->outputs.end());
    std::vector<bool> drop(g->nodes.size(), false);
    auto init_f32 = [&](const std::string &name, int64_t numel, std::vector<float> *out) {
        auto it = g->inits.find(name);
        if (it == g->inits.end() || it->second.dtype != DT_FLOAT || it->second.numel() != numel) return false;
        Value v = it->second;
        ensure_host(g, v);
        out->assign(v.h<float>(), v.h<float>() + numel);
        return true;
    };
    for (size_t j = 0; j < g->nodes.size(); ++j) {
        const NodeDef &bn = g->nodes[j];
        if (bn.op != "BatchNormalization" || bn.in.size() < 5 || attr_int(bn, "training_mode", 0)) continue;
        bool extra_out = false;
        for (size_t k = 1; k < bn.out.size(); ++k) extra_out |= !bn.out[k].empty();
        if (extra_out) continue;
        auto pi = producer.find(bn.in[0]);
        if (pi == producer.end() || uses[bn.in[0]] != 1 || outs.count(bn.in[0])) continue;
        NodeDef &cv = g->nodes[pi->second];
        if (cv.op != "Conv" || cv.in.size() < 2 || !g->inits.count(cv.in[1])) continue;
        const Value &W = g->inits.at(cv.in[1]);
        if (W.dtype != DT_FLOAT || W.shape.size() != 4) continue;
        const int64_t M = W.shape[0], per = W.numel() / std::max<int64_t>(M, 1);
        std::vector<float> w, b(M, 0.0f), sc, bb, mean, var;
        const bool has_b = cv.in.size() > 2 && !cv.in[2].empty();
        if (has_b && !init_f32(cv.in[2], M, &b)) continue;
        if (!init_f32(bn.in[1], M, &sc) || !init_f32(bn.in[2], M, &bb) || !init_f32(bn.in[3], M, &mean) ||
            !init_f32(bn.in[4], M, &var) || !init_f32(cv.in[1], W.numel(), &w))
            continue;
        const double eps = attr_float(bn, "epsilon", 1e-5f);
        std::vector<float> wf(w.size()), bf(M);
        for (int64_t m = 0; m < M; ++m) {
            const double s = (double)sc[m] / sqrt((double)var[m] + eps);
            for (int64_t k = 0; k < per; ++k) wf[m * per + k] = (float)((double)w[m * per + k] * s);
            bf[m] = (float)(((double)b[m] - (double)mean[m]) * s + (double)bb[m]);
        }
        const std::string wn = "__bnfold__/" + bn.out[0] + "/W", bname = "__bnfold__/" + bn.out[0] + "/B";
        g->inits[wn] = make_value(g, DT_FLOAT, W.shape.data(), 4, wf.data(), true);
        const int64_t bshape[1] = {M};
        g->inits[bname] = make_value(g, DT_FLOAT, bshape, 1, bf.data(), true);
        cv.in.resize(3);
        cv.in[1] = wn;
        cv.in[2] = bname;
        cv.out[0] = bn.out[0];
        drop[j] = true;
    }
    std::vector<NodeDef> kept;
    for (size_t j = 0; j < g->nodes.size(); ++j)
        if (!drop[j]) kept.push_back(std::move(g->nodes[j]));
    g->nodes.swap(kept);
}

// Layout pass: the values of a conv chain that may be stored NHWC.  A
// producer -- a Conv step, or a MaxPool --
// may write NHWC when every reader of its output takes NHWC: a Conv step
// reading it as input X (C % 32 == 0, <= 63 taps, group 1: the NHWC gather),
// a Conv step marked itself reading it as its residual, a marked MaxPool, or
// a ReduceSum/Mean/Max over axes {2, 3}.  Anything else, or being a graph
// output, keeps it NCHW.  The marks are permissions: the layout a value got
// travels with it (Value::nhwc), and lookup() converts for any other reader.
// With NHWC between them, the convs gather 16-byte rows and store their
// tiles by TMA; a 1x1 conv needs no transposed copy of its input.
// LONNX_CONV_NHWC=0 turns the pass off.
void mark_nhwc(lonnx_graph *g) {
    g->nhwc_vals.clear();
    static const bool off = getenv("LONNX_CONV_NHWC") && getenv("LONNX_CONV_NHWC")[0] == '0';
    if (off) return;
    enum Role { R_CONV_X, R_CONV_RES, R_POOL, R_REDUCE_HW, R_OTHER };
    struct Use { int step; Role role; };
    // a small-network chain step runs its sub-steps one by one unless the
    // whole chain fits one kernel (batch 1, small): its sub-steps are the
    // readers and producers (when the chain kernel runs, it reads its input
    // through lookup() and writes NCHW, which every marked reader takes too)
    std::vector<const Step *> flat;
    for (const Step &st : g->steps) {
        if (st.kind == S_TINY)
            for (const Step &t : st.sub) flat.push_back(&t);
        else
            flat.push_back(&st);
    }
    const int ns = (int)flat.size();
    std::map<std::string, std::vector<Use>> uses;
    std::vector<std::string> out(ns);       // the candidate producer's output, or empty
    std::vector<char> x_ok(ns, 0), mark(ns, 0);
    auto conv_x_ok = [&](const NodeDef &c) {
        if (c.in.size() < 2 || !g->inits.count(c.in[1])) return false;
        const Value &W = g->inits.at(c.in[1]);
        if (W.dtype != DT_FLOAT || W.shape.size() != 4) return false;
        if (const Attr *a = c.get("group"); a && g->honor_conv_attrs && a->i != 1) return false;
        const int64_t C = W.shape[1], taps = W.shape[2] * W.shape[3];
        return C % 32 == 0 && taps <= 63;
    };
    auto reduce_hw = [&](const NodeDef &n) {
        if (n.op != "ReduceMean" && n.op != "ReduceSum" && n.op != "ReduceMax") return false;
        std::vector<int64_t> axes;
        if (n.op == "ReduceMean" && g->opset < 13) {
            if (const Attr *a = n.get("axes")) axes = a->ints;
        } else if (n.in.size() > 1 && !n.in[1].empty()) {
            auto it = g->inits.find(n.in[1]);
            if (it == g->inits.end()) return false;
            Value v = it->second;
            ensure_host(g, v);
            if (v.dtype != DT_INT64) return false;
            axes.assign(v.h<int64_t>(), v.h<int64_t>() + v.numel());
        } else if (const Attr *a = n.get("axes")) {
            axes = a->ints;
        }
        std::set<int64_t> ax;
        for (auto a : axes) ax.insert(a < 0 ? a + 4 : a);
        return ax == std::set<int64_t>{2, 3};
    };
    for (int si = 0; si < ns; ++si) {
        const Step &st = *flat[si];
        if (st.kind == S_CONV) {
            const NodeDef &c = g->nodes[st.nodes[0]];
            x_ok[si] = conv_x_ok(c);
            uses[c.in.at(0)].push_back({si, x_ok[si] ? R_CONV_X : R_OTHER});
            if (!st.b.empty() && !g->inits.count(st.b)) uses[st.b].push_back({si, R_CONV_RES});
            out[si] = st.y;
            mark[si] = 1;
            continue;
        }
        if (st.kind == S_NODE && st.nodes.size() == 1) {
            const NodeDef &n = g->nodes[st.nodes[0]];
            if (n.op == "MaxPool" && !n.in.empty() && !n.out.empty()) {
                uses[n.in[0]].push_back({si, R_POOL});
                out[si] = n.out[0];
                mark[si] = 1;
                continue;
            }
            if (reduce_hw(n) && !n.in.empty()) {
                uses[n.in[0]].push_back({si, R_REDUCE_HW});
                for (size_t k = 1; k < n.in.size(); ++k) uses[n.in[k]].push_back({si, R_OTHER});
                continue;
            }
        }
        for (int i : st.nodes)
            for (auto &in : g->nodes[i].in) uses[in].push_back({si, R_OTHER});
    }
    const std::set<std::string> outs(g->outputs.begin(), g->outputs.end());
    for (bool changed = true; changed;) {
        changed = false;
        for (int si = 0; si < ns; ++si) {
            if (!mark[si]) continue;
            bool ok = !outs.count(out[si]);
            for (const Use &u : uses[out[si]]) {
                if (u.role == R_CONV_X || u.role == R_REDUCE_HW) continue;
                if (u.role == R_CONV_RES && mark[u.step] && x_ok[u.step]) continue;
                if (u.role == R_POOL && mark[u.step]) continue;
                ok = false;
            }
            if (!ok) { mark[si] = 0; changed = true; }
        }
    }
    for (int si = 0; si < ns; ++si)
        if (mark[si]) g->nhwc_vals.insert(out[si]);
}

void build_steps(lonnx_graph *g, bool fuse) {
    g->steps.clear();
    if (fuse) fold_batchnorm(g);
    const int n = (int)g->nodes.size();
    if (!fuse) {
        for (int i = 0; i < n; ++i) {
            Step s;
            s.nodes = {i};
            g->steps.push_back(s);
        }
        return;
    }
    Matcher m(g);
    // pass 1: find fusable groups; each node joins at most one group
    std::vector<Step> groups;
    std::vector<int> owner(n, -1);
    auto claim = [&](Step &st) {
        for (int x : st.nodes)
            if (m.used[x]) return false;
        for (int x : st.nodes) { m.used[x] = true; owner[x] = (int)groups.size(); }
        groups.push_back(st);
        return true;
    };
    for (int i = 0; i < n; ++i) {
        if (m.used[i]) continue;
        Step st;
        std::vector<int> hn;
        if (match_attn(m, i, st, hn)) { claim(st); continue; }
    }
    for (int i = 0; i < n; ++i) {
        if (m.used[i]) continue;
        Step st;
        if (match_gemm(m, i, st) || match_gemm_onnx(m, i, st)) { claim(st); continue; }
    }
    for (int i = 0; i < n; ++i) {
        if (m.used[i]) continue;
        Step st;
        if (match_ln(m, i, st)) { claim(st); continue; }
    }
    for (int i = 0; i < n; ++i) {
        if (m.used[i]) continue;
        Step st;
        if (match_conv(m, i, st)) { claim(st); continue; }
    }
    // weight re-layout for GEMM groups: W [K, N] -> [N, K]
    for (auto &st : groups) {
        if (st.kind != S_GEMM) continue;
        const Value &W = g->inits.at(st.a);
        st.wt = std::make_shared<DevBuf>(g->ctx, (size_t)st.N * st.K * 4);
        st.wlo = std::make_shared<DevBuf>(g->ctx, (size_t)st.N * st.K * 4);
        ck(split_tf32_nk(g->ctx, (const float *)W.dptr(), (float *)st.wt->p, (float *)st.wlo->p, st.K, st.N,
                         st.wtrans));
        if (st.b.empty()) {
            st.bias = nullptr;
        } else if (st.bias_beta == 1.0f) {
            st.bias = g->inits.at(st.b).buf;
        } else {
            Value B = g->inits.at(st.b);
            ensure_host(g, B);
            std::vector<float> scaled(st.N);
            for (int j = 0; j < st.N; ++j) scaled[j] = st.bias_beta * B.h<float>()[j];
            st.bias = std::make_shared<DevBuf>(g->ctx, (size_t)st.N * 4);
            ck(lonnx_memcpy_h2d(g->ctx, st.bias->p, scaled.data(), (size_t)st.N * 4));
        }
    }
    // conv weights [M, C, kh, kw] = [M, K] -> tf32 hi / lo [M, ldk] once
    for (auto &st : groups) {
        if (st.kind != S_CONV) continue;
        const NodeDef &c = g->nodes[st.nodes[0]];
        if (c.in.size() < 2 || !g->inits.count(c.in[1])) continue;
        const Value &W = g->inits.at(c.in[1]);
        if (W.dtype != DT_FLOAT || W.shape.size() != 4) continue;
        const int M = (int)W.shape[0], K = (int)(W.shape[1] * W.shape[2] * W.shape[3]), ldk = (K + 3) & ~3;
        st.wt = std::make_shared<DevBuf>(g->ctx, (size_t)M * ldk * 4);
        st.wlo = std::make_shared<DevBuf>(g->ctx, (size_t)M * ldk * 4);
        const int C = (int)W.shape[1], kh = (int)W.shape[2], kw = (int)W.shape[3];
        st.w_tapmajor = conv_nhwc_ok(C, kh, kw) ? 1 : 0;
        if (st.w_tapmajor)
            ck(split_rows_tapmajor(g->ctx, (const float *)W.dptr(), (float *)st.wt->p, (float *)st.wlo->p, M, C, kh * kw));
        else
            ck(split_pad_rows(g->ctx, (const float *)W.dptr(), (float *)st.wt->p, (float *)st.wlo->p, M, K, ldk));
    }
    // QKV merge: three GEMM groups on one input feeding one attention group
    for (auto &at : groups) {
        if (at.kind != S_ATTN) continue;
        int gq = -1, gk = -1, gv = -1;
        for (size_t j = 0; j < groups.size(); ++j) {
            if (groups[j].kind != S_GEMM || groups[j].epi != LONNX_EPI_NONE) continue;
            if (groups[j].y == at.q) gq = (int)j;
            if (groups[j].y == at.k) gk = (int)j;
            if (groups[j].y == at.v) gv = (int)j;
        }
        if (gq < 0 || gk < 0 || gv < 0) continue;
        Step &Q = groups[gq], &Kq = groups[gk], &V = groups[gv];
        if (Q.x != Kq.x || Q.x != V.x || Q.K != Kq.K || Q.K != V.K || Q.N != Kq.N || Q.N != V.N) continue;
        const int H = Q.N, K = Q.K;
        auto wt = std::make_shared<DevBuf>(g->ctx, (size_t)3 * H * K * 4);
        auto wlo = std::make_shared<DevBuf>(g->ctx, (size_t)3 * H * K * 4);
        auto bs = std::make_shared<DevBuf>(g->ctx, (size_t)3 * H * 4);
        Step *parts[3] = {&Q, &Kq, &V};
        for (int p = 0; p < 3; ++p) {
            ck(lonnx_memcpy_d2d(g->ctx, (float *)wt->p + (size_t)p * H * K, parts[p]->wt->p, (size_t)H * K * 4));
            ck(lonnx_memcpy_d2d(g->ctx, (float *)wlo->p + (size_t)p * H * K, parts[p]->wlo->p, (size_t)H * K * 4));
            ck(lonnx_memcpy_d2d(g->ctx, (float *)bs->p + (size_t)p * H, parts[p]->bias->p, (size_t)H * 4));
        }
        Q.wt = wt;
        Q.wlo = wlo;
        Q.bias = bs;
        Q.N = 3 * H;
        Q.y = "__qkv__" + at.y;
        for (int x : Kq.nodes) Q.nodes.push_back(x);
        for (int x : V.nodes) Q.nodes.push_back(x);
        Kq.kind = V.kind = S_NODE;
        Kq.nodes.clear();
        V.nodes.clear();
        at.qkv_packed = true;
        at.qkv = Q.y;
    }
    // emit steps in order of each group's last node (all its inputs are then available)
    std::vector<std::pair<int, int>> order;  // (position, group or -1-node)
    for (size_t j = 0; j < groups.size(); ++j) {
        if (groups[j].nodes.empty()) continue;
        int pos = *std::max_element(groups[j].nodes.begin(), groups[j].nodes.end());
        if (groups[j].kind == S_GEMM && !groups[j].y.empty() && groups[j].y.rfind("__qkv__", 0) == 0) {
            // the packed QKV GEMM must run before its attention: place it at its first node
            pos = *std::min_element(groups[j].nodes.begin(), groups[j].nodes.end());
        }
        order.push_back({pos, (int)j});
    }
    for (int i = 0; i < n; ++i)
        if (!m.used[i]) order.push_back({i, -1 - i});
    std::stable_sort(order.begin(), order.end(), [](auto &a, auto &b) { return a.first < b.first; });
    for (auto &o : order) {
        if (o.second >= 0) {
            Step s = groups[o.second];
            std::sort(s.nodes.begin(), s.nodes.end());
            g->steps.push_back(s);
        } else {
            Step s;
            s.nodes = {-1 - o.second};
            g->steps.push_back(s);
        }
    }
    // small-network chains: consecutive Conv / MaxPool / Reshape / MatMul /
    // Add steps starting at a Conv, each taking the previous step's output,
    // which nothing else uses, as its input.  Whether a chain runs as one
    // kernel is decided at run time (batch 1, sizes; exec_tiny_step).
    auto out_of = [&](const Step &st) -> std::string {
        if (st.kind == S_CONV) return st.y;
        if (st.kind == S_NODE && st.nodes.size() == 1 && !g->nodes[st.nodes[0]].out.empty())
            return g->nodes[st.nodes[0]].out[0];
        return std::string();
    };
    auto chain_op = [&](const Step &st) {
        if (st.kind == S_CONV) return true;
        if (st.kind != S_NODE || st.nodes.size() != 1) return false;
        const std::string &op = g->nodes[st.nodes[0]].op;
        return op == "MaxPool" || op == "Reshape" || op == "MatMul" || op == "Add";
    };
    auto takes = [&](const Step &st, const std::string &prev) {
        if (prev.empty()) return false;
        const int cons = m.only_consumer(prev);  // -1 as well for a graph output
        if (cons < 0 || std::find(st.nodes.begin(), st.nodes.end(), cons) == st.nodes.end()) return false;
        if (st.kind == S_CONV) return g->nodes[st.nodes[0]].in.at(0) == prev;
        const NodeDef &nd = g->nodes[st.nodes[0]];
        if (nd.op == "Add") return nd.in.size() == 2 && ((nd.in[0] == prev) != (nd.in[1] == prev));
        return !nd.in.empty() && nd.in[0] == prev;
    };
    std::vector<Step> chained;
    for (size_t i = 0; i < g->steps.size();) {
        size_t j = i + 1;
        if (g->steps[i].kind == S_CONV)
            while (j < g->steps.size() && chain_op(g->steps[j]) && takes(g->steps[j], out_of(g->steps[j - 1]))) ++j;
        if (j - i >= 3) {
            Step t;
            t.kind = S_TINY;
            for (size_t k = i; k < j; ++k) {
                t.sub.push_back(g->steps[k]);
                for (int x : g->steps[k].nodes) t.nodes.push_back(x);
            }
            chained.push_back(t);
        } else {
            for (size_t k = i; k < j; ++k) chained.push_back(g->steps[k]);
        }
        i = j;
    }
    g->steps.swap(chained);
    mark_nhwc(g);
}

// The chain of a TINY step as one kernel, planned from the run-time shapes;
// false (nothing run) when a step of it would not take the per-step kernels
// that tiny.cu reproduces, or an activation does not fit.
bool exec_tiny_step(lonnx_graph *g, const Step &s) {
    static const bool off = getenv("LONNX_TINY_CHAIN") && getenv("LONNX_TINY_CHAIN")[0] == '0';
    if (off || s.sub.empty() || s.sub[0].kind != S_CONV) return false;
    const NodeDef &c0 = g->nodes[s.sub[0].nodes[0]];
    // (an NHWC-stored input: a conv chain of a larger batch, run step by step)
    Value x = lookup_raw(g, c0.in.at(0));
    if (x.nhwc || x.dtype != DT_FLOAT || x.shape.size() != 4 || x.shape[0] != 1) return false;
    TinyProg p{};
    std::vector<int64_t> cur = x.shape;
    auto numel = [](const std::vector<int64_t> &v) {
        int64_t n = 1;
        for (auto d : v) n *= d;
        return n;
    };
    p.in_elems = (int)std::min<int64_t>(numel(cur), 1 << 30);
    if (numel(cur) > TINY_MAX_SMEM_FLOATS) return false;
    int64_t maxe = numel(cur);
    std::vector<Value> keep;  // device buffers the kernel reads
    std::string prev;         // the previous sub-step's output
    for (const Step &st : s.sub) {
        if (p.n >= TINY_MAX_LAYERS) return false;
        TinyLayer &L = p.L[p.n];
        if (st.kind == S_CONV) {
            const NodeDef &c = g->nodes[st.nodes[0]];
            Value w = lookup(g, c.in.at(1));
            if (w.dtype != DT_FLOAT) return false;
            const ConvGeom q = conv_geom(g, c, cur, w.shape);
            const int64_t total = (int64_t)q.N * q.M * q.Ho * q.Wo, K = (int64_t)q.C * q.kh * q.kw;
            if (q.N != 1 || q.group != 1 || total * K >= gemm_tc_min_work()) return false;  // not the direct kernel
            Value bias;
            bool has_bias = c.in.size() > 2 && !c.in[2].empty();
            if (!st.b.empty()) {  // the Add after the conv: a per-channel bias only (no residual)
                if (has_bias) return false;
                bias = lookup(g, st.b);
                if (bias.dtype != DT_FLOAT || !channel_bias_shape(bias, q.M)) return false;
                has_bias = true;
            } else if (has_bias) {
                bias = lookup(g, c.in[2]);
                if (bias.dtype != DT_FLOAT || bias.numel() != q.M) return false;
            }
            ensure_dev(g, w);
            if (has_bias) ensure_dev(g, bias);
            keep.push_back(w);
            if (has_bias) keep.push_back(bias);
            L = TinyLayer{TINY_CONV, q.C, q.H, q.W, q.M, q.kh, q.kw, q.sh, q.sw, q.pt, q.pl, q.dh, q.dw, q.Ho, q.Wo,
                          st.epi ? 1 : 0, 0, 0, (const float *)w.dptr(), has_bias ? (const float *)bias.dptr() : nullptr};
            cur = {1, q.M, q.Ho, q.Wo};
        } else if (st.kind == S_NODE && st.nodes.size() == 1) {
            const NodeDef &n = g->nodes[st.nodes[0]];
            if (n.op == "MaxPool") {
                const PoolGeom q = pool_geom(n, cur);
                L = TinyLayer{TINY_MAXPOOL, q.C, q.H, q.W, 0, q.kh, q.kw, q.sh, q.sw, q.pt, q.pl, 1, 1, q.Ho, q.Wo,
                              0, 0, 0, nullptr, nullptr};
                cur = {1, q.C, q.Ho, q.Wo};
            } else if (n.op == "Reshape") {
                cur = reshape_shape(g, n, cur);
                L = TinyLayer{};
                L.op = TINY_VIEW;
            } else if (n.op == "MatMul") {
                Value w = lookup(g, n.in.at(1));
                if (w.dtype != DT_FLOAT || w.shape.size() != 2 || cur.size() != 2 || cur[0] != 1 || cur[1] != w.shape[0])
                    return false;
                const int64_t K = w.shape[0], N = w.shape[1];
                // the path the product would take: below the tensor-core
                // threshold and small enough for k_gemm_rowdot_smem
                if (K * N >= gemm_tc_min_work() || N > 256 || (K + K * N) * 4 > 48 * 1024) return false;
                ensure_dev(g, w);
                keep.push_back(w);
                L = TinyLayer{};
                L.op = TINY_FC;
                L.K = (int)K;
                L.N = (int)N;
                L.w = (const float *)w.dptr();
                cur = {1, N};
            } else if (n.op == "Add") {
                // the bias Add right after the MatMul
                if (p.n == 0 || p.L[p.n - 1].op != TINY_FC || p.L[p.n - 1].bias) return false;
                Value b = lookup(g, n.in.at(0) == prev ? n.in.at(1) : n.in.at(0));
                const int64_t N = p.L[p.n - 1].N;
                if (b.dtype != DT_FLOAT || b.numel() != N || b.shape.size() > 2 || b.shape.back() != N) return false;
                ensure_dev(g, b);
                keep.push_back(b);
                p.L[p.n - 1].bias = (const float *)b.dptr();
                prev = n.out.at(0);
                continue;  // folded into the MatMul layer
            } else {
                return false;
            }
        } else {
            return false;
        }
        prev = st.kind == S_CONV ? st.y : g->nodes[st.nodes[0]].out.at(0);
        ++p.n;
        maxe = std::max(maxe, numel(cur));
    }
    if (p.n == 0) return false;
    p.max_elems = (int)std::min<int64_t>(maxe, 1 << 30);
    int64_t smem = 2 * maxe;  // two activation buffers, then every layer's weights
    for (int l = 0; l < p.n; ++l) {
        TinyLayer &L = p.L[l];
        L.woff = (int)std::min<int64_t>(smem, 1 << 30);
        smem += L.op == TINY_FC ? (int64_t)L.K * L.N : L.op == TINY_CONV ? (int64_t)L.M * L.C * L.kh * L.kw : 0;
    }
    if (smem > TINY_MAX_SMEM_FLOATS) return false;
    p.smem_floats = (int)smem;
    ensure_dev(g, x);
    Value y = new_dev(g, DT_FLOAT, cur);
    ck(tiny_chain(g->ctx, p, (const float *)x.dptr(), (float *)y.dptr_mut()));
    const Step &last = s.sub.back();
    g->env[last.kind == S_CONV ? last.y : g->nodes[last.nodes[0]].out.at(0)] = y;
    return true;
}

void run_step(lonnx_graph *g, const Step &s) {
    bool done = false;
    switch (s.kind) {
    case S_GEMM: done = exec_gemm_step(g, s); break;
    case S_LN: done = exec_ln_step(g, s); break;
    case S_ATTN: done = exec_attn_step(g, s); break;
    case S_CONV: done = exec_conv_step(g, s); break;
    case S_TINY:
        if (!exec_tiny_step(g, s))
            for (const Step &t : s.sub) run_step(g, t);
        return;
    default: break;
    }
    if (!done) {
        if (s.kind == S_ATTN && s.qkv_packed) fail(LONNX_E_SHAPE, "fused attention: unexpected shapes for packed QKV");
        for (int i : s.nodes) exec_node(g, g->nodes[i]);
    }
}

void run_steps(lonnx_graph *g) {
    for (auto &s : g->steps) run_step(g, s);
}

template <typename F>
int guarded(F &&f) {
    try {
        return f();
    } catch (const OpError &e) {
        return set_error(e.code, "%s", e.what());
    } catch (const std::exception &e) {
        return set_error(LONNX_E_BADARG, "%s", e.what());
    }
}

Value make_value(lonnx_graph *g, int dtype, const int64_t *shape, int rank, const void *host, bool upload) {
    if (!dtype_size(dtype)) fail(LONNX_E_UNSUPPORTED, "unsupported dtype " + std::to_string(dtype));
    if (rank < 0 || rank > 8) fail(LONNX_E_BADARG, "rank out of range");
    Value v;
    v.dtype = dtype;
    v.shape.assign(shape, shape + rank);
    const size_t bytes = v.bytes();
    if (dtype != DT_FLOAT || v.numel() <= 4096) {
        v.host = std::make_shared<std::vector<uint8_t>>(bytes);
        if (bytes) memcpy(v.host->data(), host, bytes);
    }
    if (upload || dtype == DT_FLOAT) {
        v.buf = std::make_shared<DevBuf>(g->ctx, bytes);
        if (bytes) ck(lonnx_memcpy_h2d(g->ctx, v.buf->p, host, bytes));
    }
    return v;
}

void release_capture(lonnx_graph *g) {
    if (g->exec) {
        cudaStreamSynchronize(g->ctx->stream);
        cudaGraphExecDestroy(g->exec);
        g->exec = nullptr;
    }
    g->captured_outputs.clear();
    for (void *p : g->held) ctx_free(g->ctx, p);
    g->held.clear();
}

}  // namespace

extern "C" {

LONNX_API int lonnx_graph_capture(lonnx_graph *g) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&]() -> int {
        if (!g->prepared) build_steps(g, false), g->prepared = true;
        release_capture(g);
        lonnx_ctx *c = g->ctx;
        g->env.clear();
        LONNX_CUDA(cudaStreamSynchronize(c->stream));
        LONNX_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
        c->capturing = true;
        int err = LONNX_OK;
        std::string msg;
        try {
            run_steps(g);
            for (auto &o : g->outputs)
                if (!has_value(g, o)) fail(LONNX_E_BADARG, "graph output " + o + " was not produced");
        } catch (const OpError &e) {
            err = e.code;
            msg = e.what();
        }
        cudaGraph_t graph = nullptr;
        cudaError_t ce = cudaStreamEndCapture(c->stream, &graph);
        c->capturing = false;
        g->held.swap(c->capture_hold);
        c->capture_hold.clear();
        if (err) {
            if (graph) cudaGraphDestroy(graph);
            g->env.clear();
            release_capture(g);
            fail(err, "capture failed: " + msg);
        }
        if (ce != cudaSuccess) {
            cudaGetLastError();
            release_capture(g);
            fail(LONNX_E_CUDA, std::string("capture failed: ") + cudaGetErrorString(ce));
        }
        ce = cudaGraphInstantiate(&g->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ce != cudaSuccess) {
            cudaGetLastError();
            release_capture(g);
            fail(LONNX_E_CUDA, std::string("graph instantiate failed: ") + cudaGetErrorString(ce));
        }
        for (auto &o : g->outputs) g->captured_outputs[o] = lookup(g, o);
        g->env = g->captured_outputs;
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_replay(lonnx_graph *g) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    if (!g->exec) return set_error(LONNX_E_BADARG, "graph was not captured");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    LONNX_CUDA(cudaGraphLaunch(g->exec, g->ctx->stream));
    g->ctx->launches++;
    g->env = g->captured_outputs;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_create(lonnx_ctx *ctx, lonnx_graph **out) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!out) return set_error(LONNX_E_BADARG, "null output");
    lonnx_graph *g = new lonnx_graph();
    g->ctx = ctx;
    *out = g;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_destroy(lonnx_graph *g) {
    if (!g) return LONNX_OK;
    device_guard(g->ctx);
    cudaStreamSynchronize(g->ctx->stream);
    release_capture(g);
    delete g;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_add_initializer(lonnx_graph *g, const char *name, int dtype, const int64_t *shape, int rank,
                                          const void *host_data) {
    if (!g || !name) return set_error(LONNX_E_BADARG, "null argument");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&] {
        // every initializer is uploaded once; small ones also keep a host copy
        g->inits[name] = make_value(g, dtype, shape, rank, host_data, true);
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_add_node(lonnx_graph *g, const char *op, const char *const *inputs, int n_in,
                                   const char *const *outputs, int n_out) {
    if (!g || !op || n_in < 0 || n_out < 0) return set_error(LONNX_E_BADARG, "bad node");
    NodeDef n;
    n.op = op;
    for (int i = 0; i < n_in; ++i) n.in.push_back(inputs[i] ? inputs[i] : "");
    for (int i = 0; i < n_out; ++i) n.out.push_back(outputs[i] ? outputs[i] : "");
    g->nodes.push_back(n);
    g->prepared = false;
    return LONNX_OK;
}

static NodeDef *last_node(lonnx_graph *g) { return (g && !g->nodes.empty()) ? &g->nodes.back() : nullptr; }

LONNX_API int lonnx_graph_attr_int(lonnx_graph *g, const char *name, int64_t v) {
    NodeDef *n = last_node(g);
    if (!n || !name) return set_error(LONNX_E_BADARG, "no node");
    Attr a;
    a.kind = 1;
    a.i = v;
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_set_opset(lonnx_graph *g, int opset) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    g->opset = opset;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_attr_ints(lonnx_graph *g, const char *name, const int64_t *v, int cnt) {
    NodeDef *n = last_node(g);
    if (!n || !name || cnt < 0) return set_error(LONNX_E_BADARG, "no node");
    Attr a;
    a.kind = 2;
    a.ints.assign(v, v + cnt);
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_attr_float(lonnx_graph *g, const char *name, float v) {
    NodeDef *n = last_node(g);
    if (!n || !name) return set_error(LONNX_E_BADARG, "no node");
    Attr a;
    a.kind = 3;
    a.f = v;
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_attr_string(lonnx_graph *g, const char *name, const char *v) {
    NodeDef *n = last_node(g);
    if (!n || !name || !v) return set_error(LONNX_E_BADARG, "no node");
    Attr a;
    a.kind = 4;
    a.s = v;
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_attr_floats(lonnx_graph *g, const char *name, const float *v, int cnt) {
    NodeDef *n = last_node(g);
    if (!n || !name || cnt < 0 || (cnt && !v)) return set_error(LONNX_E_BADARG, "no node");
    Attr a;
    a.kind = 5;
    a.floats.assign(v, v + cnt);
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_attr_tensor(lonnx_graph *g, const char *name, int dtype, const int64_t *shape, int rank,
                                      const void *data) {
    NodeDef *n = last_node(g);
    if (!n || !name || rank < 0 || rank > 8 || (rank && !shape)) return set_error(LONNX_E_BADARG, "no node");
    if (!dtype_size(dtype)) return set_error(LONNX_E_UNSUPPORTED, "unsupported dtype %d", dtype);
    Attr a;
    a.kind = 6;
    a.tdtype = dtype;
    a.tshape.assign(shape, shape + rank);
    int64_t cnt = 1;
    for (auto d : a.tshape) {
        if (d < 0) return set_error(LONNX_E_BADARG, "negative dimension");
        cnt *= d;
    }
    const size_t bytes = (size_t)cnt * dtype_size(dtype);
    if (bytes && !data) return set_error(LONNX_E_BADARG, "null tensor data");
    a.tdata.assign((const uint8_t *)data, (const uint8_t *)data + bytes);
    n->attrs[name] = a;
    return LONNX_OK;
}

LONNX_API int lonnx_graph_add_output(lonnx_graph *g, const char *name) {
    if (!g || !name) return set_error(LONNX_E_BADARG, "null argument");
    g->outputs.push_back(name);
    return LONNX_OK;
}

LONNX_API int lonnx_graph_prepare(lonnx_graph *g, int flags) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&] {
        g->honor_conv_attrs = (flags & 2) != 0;
        build_steps(g, (flags & 1) != 0);
        g->prepared = true;
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_set_input(lonnx_graph *g, const char *name, int dtype, const int64_t *shape, int rank,
                                    const void *host_data) {
    if (!g || !name) return set_error(LONNX_E_BADARG, "null argument");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&] {
        g->inputs[name] = make_value(g, dtype, shape, rank, host_data, true);
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_set_input_device(lonnx_graph *g, const char *name, int dtype, const int64_t *shape, int rank,
                                           const void *dev_data) {
    if (!g || !name) return set_error(LONNX_E_BADARG, "null argument");
    return guarded([&] {
        if (!dtype_size(dtype) || rank < 0 || rank > 8) fail(LONNX_E_BADARG, "bad input description");
        Value v;
        v.dtype = dtype;
        v.shape.assign(shape, shape + rank);
        v.ext = dev_data;
        g->inputs[name] = v;
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_execute(lonnx_graph *g) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&] {
        if (!g->prepared) build_steps(g, false), g->prepared = true;
        g->env.clear();
        run_steps(g);
        for (auto &o : g->outputs)
            if (!has_value(g, o)) fail(LONNX_E_BADARG, "graph output " + o + " was not produced");
        // keep only the outputs; intermediates go back to the allocator
        std::map<std::string, Value> keep;
        for (auto &o : g->outputs) keep[o] = lookup(g, o);
        g->env.swap(keep);
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_output_shape(lonnx_graph *g, const char *name, int64_t *shape, int *rank) {
    if (!g || !name || !rank) return set_error(LONNX_E_BADARG, "null argument");
    return guarded([&] {
        const Value &v = lookup(g, name);
        *rank = (int)v.shape.size();
        for (size_t i = 0; i < v.shape.size(); ++i) shape[i] = v.shape[i];
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_output_dtype(lonnx_graph *g, const char *name, int *dtype) {
    if (!g || !name || !dtype) return set_error(LONNX_E_BADARG, "null argument");
    return guarded([&] {
        *dtype = lookup(g, name).dtype;
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_output_device(lonnx_graph *g, const char *name, const void **dev) {
    if (!g || !name || !dev) return set_error(LONNX_E_BADARG, "null argument");
    return guarded([&] {
        Value v = lookup(g, name);
        ensure_dev(g, v);
        g->env[name] = v;
        *dev = v.dptr();
        return LONNX_OK;
    });
}

LONNX_API int lonnx_graph_get_output(lonnx_graph *g, const char *name, void *host, size_t bytes) {
    if (!g || !name) return set_error(LONNX_E_BADARG, "null argument");
    int rc = device_guard(g->ctx);
    if (rc) return rc;
    return guarded([&] {
        const Value &v = lookup(g, name);
        if (bytes != v.bytes()) fail(LONNX_E_BADARG, "output buffer size mismatch");
        if (v.on_dev()) ck(lonnx_memcpy_d2h(g->ctx, host, v.dptr(), bytes));
        else if (bytes) memcpy(host, v.host->data(), bytes);
        return lonnx_sync(g->ctx);
    });
}

LONNX_API int lonnx_graph_reset(lonnx_graph *g) {
    if (!g) return set_error(LONNX_E_BADARG, "null graph");
    release_capture(g);
    g->env.clear();
    g->inputs.clear();
    return LONNX_OK;
}

LONNX_API int lonnx_graph_num_steps(lonnx_graph *g) { return g ? (int)g->steps.size() : 0; }

}  // extern "C"
