// Orchestration of one MoE layer call and the C ABI (include/sparsemoe_b200.h).
//
// Stage order on the caller's stream (all asynchronous):
//   router_topk -> dispatch (count, scan, assign+gather) -> up/gate GEMM with
//   fused SwiGLU -> down GEMM -> combine.
// The library owns one small device scratch block per device (routing tables,
// status word), grown on demand and freed by moe_release(); every large
// buffer comes from the caller's MoEArgs, as in the reference
// (inputs/data.cu:199-524 allocates, kernels/launcher.h:21 only launches).
#include "moe_internal.h"
#include "../../include/config.h"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

namespace moe {

namespace {
thread_local std::string g_error;
// Optional per-stage timing events (moe_set_stage_events), per host thread.
constexpr int kStageEvents = 6;
thread_local cudaEvent_t g_stage_ev[kStageEvents] = {};
thread_local bool g_stage_on = false;
std::mutex g_mu;
constexpr int kMaxDevices = 64;
struct DeviceState {
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int* status = nullptr;  // status word of the last call (inside ws)
    int num_sms = 0;
    int cc_major = -1;
};
DeviceState g_dev[kMaxDevices];

MoeDims default_dims() {
    MoeDims d{};
    d.num_batches = num_batches;
    d.tokens = N;
    d.d_model = d_model;
    d.d_ff = up_proj_dim * d_model;
    d.num_experts = num_experts;
    d.top_k = k;
    d.capacity_factor = capacity_factor;
    d.cap = 0;
    d.dtype = MOE_DTYPE_F16;
    d.router_dtype = MOE_ROUTER_SAME;
    d.router_bias = nullptr;
    d.output_16 = nullptr;
    return d;
}
MoeDims g_solve_dims = default_dims();

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
}  // namespace

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
}

size_t workspace_header_bytes() { return 256 + 5 * align256(sizeof(int) * kMaxGroups); }

// Per-row activation scales: FP8 one per 1x128 block of x / h; INT8_CHANNEL one
// per row of x and one per 1x128 block of h.
size_t scale_bytes(const Shape& s, int dim) {
    if (s.dtype == MOE_DTYPE_FP8_BLOCK || (s.dtype == MOE_DTYPE_INT8_CHANNEL && dim == s.f))
        return align256(sizeof(float) * (size_t)s.rows_capacity() * (dim / 128));
    if (s.dtype == MOE_DTYPE_INT8_CHANNEL) return align256(sizeof(float) * (size_t)s.rows_capacity());
    return 0;
}

size_t router_scratch_bytes(const Shape& s) {
    const size_t nb = (size_t)(s.d + kRouterBlockJ - 1) / kRouterBlockJ;
    return router_blocked(s) ? align256(sizeof(float) * nb * (size_t)s.T() * s.E) : 0;
}

size_t workspace_bytes(const Shape& s) {
    const size_t routes = (size_t)s.T() * s.k;
    const size_t chunk_tab = (size_t)s.B * s.chunks() * s.E;
    return workspace_header_bytes() + align256(sizeof(int) * routes) + 2 * align256(sizeof(int) * chunk_tab) +
           align256(sizeof(int) * (size_t)s.B * s.E) + 2 * align256(sizeof(int) * s.E) + scale_bytes(s, s.d) +
           scale_bytes(s, s.f) + router_scratch_bytes(s);
}

void carve_workspace(void* base, const Shape& s, Workspace* ws) {
    uint8_t* p = static_cast<uint8_t*>(base);
    const size_t routes = (size_t)s.T() * s.k;
    const size_t chunk_tab = (size_t)s.B * s.chunks() * s.E;
    ws->status = reinterpret_cast<int*>(p);       p += 256;
    ws->grp_rows = reinterpret_cast<int*>(p);     p += align256(sizeof(int) * kMaxGroups);
    ws->grp_start = reinterpret_cast<int*>(p);    p += align256(sizeof(int) * kMaxGroups);
    ws->grp_weight = reinterpret_cast<int*>(p);   p += align256(sizeof(int) * kMaxGroups);
    ws->grp_out_rank = reinterpret_cast<int*>(p); p += align256(sizeof(int) * kMaxGroups);
    ws->grp_out_row = reinterpret_cast<int*>(p);  p += align256(sizeof(int) * kMaxGroups);
    ws->route_slot = reinterpret_cast<int*>(p);   p += align256(sizeof(int) * routes);
    ws->chunk_count = reinterpret_cast<int*>(p);  p += align256(sizeof(int) * chunk_tab);
    ws->chunk_base = reinterpret_cast<int*>(p);   p += align256(sizeof(int) * chunk_tab);
    ws->row_base = reinterpret_cast<int*>(p);     p += align256(sizeof(int) * (size_t)s.B * s.E);
    ws->expert_rows = reinterpret_cast<int*>(p);  p += align256(sizeof(int) * s.E);
    ws->expert_start = reinterpret_cast<int*>(p); p += align256(sizeof(int) * s.E);
    ws->a_scale = scale_bytes(s, s.d) ? reinterpret_cast<float*>(p) : nullptr;
    p += scale_bytes(s, s.d);
    ws->h_scale = scale_bytes(s, s.f) ? reinterpret_cast<float*>(p) : nullptr;
    p += scale_bytes(s, s.f);
    ws->router_logits = router_scratch_bytes(s) ? reinterpret_cast<float*>(p) : nullptr;
}

namespace {

int cuda_fail(cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return MOE_ERR_CUDA;
}

// Shape checks shared by every entry point; with bind_check, also that the
// format's MoeDims pointers (weight scales) are set.
int make_shape(const MoeDims* d, Shape* s, bool bind_check = true) {
    if (!d) { set_error("dims is null"); return MOE_ERR_INVALID_ARG; }
    if (d->num_batches < 0 || d->tokens < 0 || d->d_model <= 0 || d->d_ff <= 0 || d->num_experts <= 0 ||
        d->top_k <= 0) {
        set_error("non-positive dimension");
        return MOE_ERR_INVALID_ARG;
    }
    if (d->top_k > 32 || d->top_k > d->num_experts) {
        set_error("top_k=%d must be <= 32 and <= num_experts=%d", d->top_k, d->num_experts);
        return MOE_ERR_INVALID_ARG;
    }
    if (d->num_experts % 8 != 0 || d->num_experts > 256) {
        set_error("num_experts=%d: this build needs a multiple of 8, <= 256", d->num_experts);
        return MOE_ERR_UNSUPPORTED;
    }
    if (d->d_model % 256 != 0 || d->d_ff % 128 != 0) {
        set_error("d_model=%d must be a multiple of 256 and d_ff=%d of 128", d->d_model, d->d_ff);
        return MOE_ERR_UNSUPPORTED;
    }
    if (d->dtype != MOE_DTYPE_F16 && d->dtype != MOE_DTYPE_BF16 && d->dtype != MOE_DTYPE_INT8 &&
        d->dtype != MOE_DTYPE_FP8_BLOCK && d->dtype != MOE_DTYPE_W4A16 && d->dtype != MOE_DTYPE_INT8_CHANNEL &&
        d->dtype != MOE_DTYPE_NVFP4 && d->dtype != MOE_DTYPE_INT4_PTX && d->dtype != MOE_DTYPE_FP8) {
        set_error("dtype %d not supported by this entry point", d->dtype);
        return MOE_ERR_UNSUPPORTED;
    }
    if (d->router_dtype != MOE_ROUTER_SAME && d->router_dtype != MOE_ROUTER_F32) {
        set_error("router_dtype %d unknown", d->router_dtype);
        return MOE_ERR_INVALID_ARG;
    }
    s->B = d->num_batches;
    s->N = d->tokens;
    s->d = d->d_model;
    s->f = d->d_ff;
    s->E = d->num_experts;
    s->k = d->top_k;
    s->dtype = d->dtype;
    s->router_dtype = d->router_dtype;
    s->act_bf16 = d->dtype == MOE_DTYPE_BF16 || d->dtype == MOE_DTYPE_FP8_BLOCK || d->dtype == MOE_DTYPE_W4A16 ||
                  d->dtype == MOE_DTYPE_INT8_CHANNEL || d->dtype == MOE_DTYPE_NVFP4;
    if (bind_check && d->dtype == MOE_DTYPE_NVFP4 && (!d->w4_scale_gate || !d->w4_scale_up || !d->w4_scale_down ||
                                        !d->fp4_global_gate || !d->fp4_global_up || !d->fp4_global_down)) {
        set_error("MOE_DTYPE_NVFP4 needs MoeDims.w4_scale_* (e4m3) and fp4_global_*");
        return MOE_ERR_INVALID_ARG;
    }
    if (bind_check && d->dtype == MOE_DTYPE_W4A16 && (!d->w4_scale_gate || !d->w4_scale_up || !d->w4_scale_down ||
                                        !d->w4_zero_gate || !d->w4_zero_up || !d->w4_zero_down)) {
        set_error("MOE_DTYPE_W4A16 needs MoeDims.w4_scale_* and w4_zero_*");
        return MOE_ERR_INVALID_ARG;
    }
    if (bind_check && (d->dtype == MOE_DTYPE_FP8_BLOCK || d->dtype == MOE_DTYPE_INT8_CHANNEL) &&
        (!d->w_scale_gate || !d->w_scale_up || !d->w_scale_down)) {
        set_error("dtype %d needs MoeDims.w_scale_gate / w_scale_up / w_scale_down", d->dtype);
        return MOE_ERR_INVALID_ARG;
    }
    if (d->cap > 0) s->cap = d->cap;
    else if (d->cap == 0) s->cap = moe_capacity(d->tokens, d->top_k, d->num_experts, d->capacity_factor);
    else s->cap = d->tokens;  // no-drop ("baseline") policy
    if (s->cap < 0) { set_error("negative capacity"); return MOE_ERR_INVALID_ARG; }
    const int64_t rows = (int64_t)s->E * s->B * s->cap;
    if (rows >= (int64_t)1 << 31 || (int64_t)s->E * s->f >= (int64_t)1 << 31 ||
        (int64_t)s->E * s->d >= (int64_t)1 << 31) {
        set_error("problem too large for 32-bit tile coordinates");
        return MOE_ERR_UNSUPPORTED;
    }
    return MOE_OK;
}

int device_state(DeviceState** out, int* dev_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev >= kMaxDevices) { set_error("device ordinal %d too large", dev); return MOE_ERR_INVALID_ARG; }
    DeviceState& st = g_dev[dev];
    if (st.cc_major < 0) {
        int major = 0, sms = 0;
        e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        st.cc_major = major;
        st.num_sms = sms;
    }
    if (st.cc_major != 10) {
        set_error("device %d has compute capability %d.x; the kernels are built for sm_100a only", dev,
                  st.cc_major);
        return MOE_ERR_NO_KERNEL;
    }
    *out = &st;
    *dev_out = dev;
    return MOE_OK;
}

int get_workspace(DeviceState& st, const Shape& s, Workspace* ws, bool header_only = false) {
    const size_t need = header_only ? workspace_header_bytes() : workspace_bytes(s);
    if (st.ws_bytes < need) {
        if (st.ws) {
            cudaError_t e = cudaFree(st.ws);
            st.ws = nullptr;
            st.ws_bytes = 0;
            if (e != cudaSuccess) return cuda_fail(e, "cudaFree(workspace)");
        }
        const size_t bytes = need + need / 4;
        cudaError_t e = cudaMalloc(&st.ws, bytes);
        if (e != cudaSuccess) { st.ws = nullptr; return cuda_fail(e, "cudaMalloc(workspace)"); }
        st.ws_bytes = bytes;
    }
    carve_workspace(st.ws, s, ws);
    st.status = ws->status;
    return MOE_OK;
}

// Workspace for a call: the caller's scratch (dims->scratch) when given, else
// the library's per-device block.
int resolve_workspace(DeviceState& st, int dev, const MoeDims* dims, const Shape& s, Workspace* ws,
                      bool header_only = false) {
    if (dims->scratch) {
        const size_t need = header_only ? workspace_header_bytes() : workspace_bytes(s);
        if (dims->scratch_bytes < need) {
            set_error("scratch of %zu bytes is smaller than the %zu this call needs", dims->scratch_bytes, need);
            return MOE_ERR_INVALID_ARG;
        }
        if (reinterpret_cast<uintptr_t>(dims->scratch) % 256 != 0) {
            set_error("scratch must be 256-byte aligned");
            return MOE_ERR_INVALID_ARG;
        }
        carve_workspace(dims->scratch, s, ws);
        if (dims->act_scale) ws->a_scale = dims->act_scale;
        note_status_word(dev, ws->status);
        return MOE_OK;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const int rc = get_workspace(st, s, ws, header_only);
    if (rc == MOE_OK && dims->act_scale) ws->a_scale = dims->act_scale;
    return rc;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_capacity(int tokens, int top_k, int num_experts, float cf) {
    // inputs/data.cu:392-398: (int)ceilf((float)N * (float)k / (float)E * cf), rounded up to 16.
    volatile float a = (float)tokens * (float)top_k;
    volatile float b = a / (float)num_experts;
    volatile float c = b * cf;
    const int raw = (int)ceilf(c);
    return ((raw + 15) / 16) * 16;
}

extern "C" size_t moe_workspace_bytes(const MoeDims* dims) {
    Shape s;
    if (make_shape(dims, &s, /*bind_check=*/false) != MOE_OK) return 0;
    return workspace_bytes(s);
}

extern "C" const char* moe_last_error(void) { return g_error.c_str(); }

extern "C" int moe_set_solve_dims(const MoeDims* dims) {
    Shape s;
    const int rc = make_shape(dims, &s);
    if (rc != MOE_OK) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    g_solve_dims = *dims;
    return MOE_OK;
}

extern "C" int moe_get_solve_dims(MoeDims* dims) {
    if (!dims) return MOE_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> lk(g_mu);
    *dims = g_solve_dims;
    return MOE_OK;
}

namespace moe {

int make_shape_checked(const MoeDims* dims, Shape* s) { return make_shape(dims, s); }

int check_args_16(const MoEArgs* a) { return check_args(a, MOE_DTYPE_F16); }

int check_args(const MoEArgs* a, int dtype) {
    if (!a) { set_error("args is null"); return MOE_ERR_INVALID_ARG; }
    const bool common = a->input && a->router_weights && a->selected_expert_indices && a->selected_expert_weights &&
                        a->expert_counts && a->expert_token_ids && a->expert_token_weights &&
                        a->hidden_mlp_layer_2_out && a->final_output;
    bool fmt = false;
    if (dtype == MOE_DTYPE_W4A16 || dtype == MOE_DTYPE_NVFP4)
        fmt = a->expert_up_proj_weights_int4 && a->expert_gate_proj_weights_int4 &&
              a->expert_down_proj_weights_int4 && a->per_expert_wmma_inputs && a->hidden_mlp_layer_1_out_fp16;
    else if (dtype == MOE_DTYPE_INT4_PTX)
        fmt = a->expert_up_proj_weights_int4 && a->expert_gate_proj_weights_int4 &&
              a->expert_down_proj_weights_int4 && a->per_expert_wmma_inputs_int8 && a->hidden_mlp_layer_1_out_int8;
    else if (dtype == MOE_DTYPE_FP8_BLOCK || dtype == MOE_DTYPE_FP8)
        fmt = a->expert_up_proj_weights_fp8 && a->expert_gate_proj_weights_fp8 && a->expert_down_proj_weights_fp8 &&
              a->per_expert_wmma_inputs_fp8 && a->hidden_mlp_layer_1_out_fp8;
    else if (dtype == MOE_DTYPE_INT8 || dtype == MOE_DTYPE_INT8_CHANNEL)
        fmt = a->expert_up_proj_weights_int8 && a->expert_gate_proj_weights_int8 &&
              a->expert_down_proj_weights_int8 && a->per_expert_wmma_inputs_int8 && a->hidden_mlp_layer_1_out_int8;
    else
        fmt = a->expert_up_proj_weights && a->expert_gate_proj_weights && a->expert_down_proj_weights &&
              a->per_expert_wmma_inputs && a->hidden_mlp_layer_1_out_fp16;
    if (!common || !fmt) {
        set_error("a MoEArgs buffer needed by the %s path is null",
                  dtype == MOE_DTYPE_INT8 || dtype == MOE_DTYPE_INT8_CHANNEL ? "int8"
                  : dtype == MOE_DTYPE_FP8_BLOCK || dtype == MOE_DTYPE_FP8  ? "fp8"
                  : dtype == MOE_DTYPE_INT4_PTX                             ? "int4 (packed-transposed)"
                  : dtype == MOE_DTYPE_W4A16 || dtype == MOE_DTYPE_NVFP4    ? "4-bit"
                                                                            : "16-bit");
        return MOE_ERR_INVALID_ARG;
    }
    if ((dtype == MOE_DTYPE_INT8 || dtype == MOE_DTYPE_INT4_PTX || dtype == MOE_DTYPE_FP8) &&
        !(a->scale_input_act > 0.0f && a->scale_mid_act > 0.0f)) {
        set_error("the per-tensor formats need positive scale_input_act and scale_mid_act");
        return MOE_ERR_INVALID_ARG;
    }
    return MOE_OK;
}

int current_device(int* dev, int* num_sms) {
    DeviceState* st = nullptr;
    const int rc = device_state(&st, dev);
    if (rc == MOE_OK) *num_sms = st->num_sms;
    return rc;
}

void note_status_word(int dev, int* status) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev >= 0 && dev < kMaxDevices) g_dev[dev].status = status;
}

GemmScales scales_of(const MoEArgs* a, const Shape& s) {
    GemmScales sc;
    if (s.dtype == MOE_DTYPE_INT8 || s.dtype == MOE_DTYPE_INT4_PTX || s.dtype == MOE_DTYPE_FP8) {
        sc.s_in = a->scale_input_act;
        sc.s_gate = a->scale_gate_w;
        sc.s_up = a->scale_up_w;
        sc.s_mid = a->scale_mid_act;
        sc.s_down = a->scale_down_w;
    }
    return sc;
}

struct FfnBuffers {
    void* a_rows;
    void* h_rows;
    const void *wg, *wu, *wd;
};
FfnBuffers ffn_buffers(const MoEArgs* a, const Shape& s) {
    const bool i8 = s.dtype == MOE_DTYPE_INT8 || s.dtype == MOE_DTYPE_INT8_CHANNEL;
    FfnBuffers b;
    if (s.dtype == MOE_DTYPE_W4A16 || s.dtype == MOE_DTYPE_NVFP4) {
        b.a_rows = (void*)a->per_expert_wmma_inputs;
        b.h_rows = (void*)a->hidden_mlp_layer_1_out_fp16;
        b.wg = a->expert_gate_proj_weights_int4;
        b.wu = a->expert_up_proj_weights_int4;
        b.wd = a->expert_down_proj_weights_int4;
        return b;
    }
    if (s.dtype == MOE_DTYPE_INT4_PTX) {
        // int4 values one per byte; the packed weights go to the GEMM as they are
        b.a_rows = (void*)a->per_expert_wmma_inputs_int8;
        b.h_rows = (void*)a->hidden_mlp_layer_1_out_int8;
        b.wg = a->expert_gate_proj_weights_int4;
        b.wu = a->expert_up_proj_weights_int4;
        b.wd = a->expert_down_proj_weights_int4;
        return b;
    }
    if (s.dtype == MOE_DTYPE_FP8_BLOCK || s.dtype == MOE_DTYPE_FP8) {
        b.a_rows = (void*)a->per_expert_wmma_inputs_fp8;
        b.h_rows = (void*)a->hidden_mlp_layer_1_out_fp8;
        b.wg = a->expert_gate_proj_weights_fp8;
        b.wu = a->expert_up_proj_weights_fp8;
        b.wd = a->expert_down_proj_weights_fp8;
        return b;
    }
    b.a_rows = i8 ? (void*)a->per_expert_wmma_inputs_int8 : (void*)a->per_expert_wmma_inputs;
    b.h_rows = i8 ? (void*)a->hidden_mlp_layer_1_out_int8 : (void*)a->hidden_mlp_layer_1_out_fp16;
    b.wg = i8 ? (const void*)a->expert_gate_proj_weights_int8 : (const void*)a->expert_gate_proj_weights;
    b.wu = i8 ? (const void*)a->expert_up_proj_weights_int8 : (const void*)a->expert_up_proj_weights;
    b.wd = i8 ? (const void*)a->expert_down_proj_weights_int8 : (const void*)a->expert_down_proj_weights;
    return b;
}

#define MOE_TRY(expr, what)                                \
    do {                                                   \
        cudaError_t e_ = (expr);                           \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

cudaError_t mark_stage(int i, cudaStream_t stream) {
    return g_stage_on ? cudaEventRecord(g_stage_ev[i], stream) : cudaSuccess;
}

// The input rows the router and the gather read: MoeDims.norm_out when the
// pre-MoE RMSNorm is on (the stage that writes it: enqueue_norm).
MoEArgs routed_args(const MoEArgs* a, const MoeDims* dims) {
    MoEArgs r = *a;
    if (dims->norm_weight) r.input = static_cast<const half*>(dims->norm_out);
    return r;
}

int check_norm(const MoeDims* dims) {
    if (dims->norm_weight && !dims->norm_out) {
        set_error("MoeDims.norm_weight needs MoeDims.norm_out (device [B, N, d] for the normalised rows)");
        return MOE_ERR_INVALID_ARG;
    }
    if (dims->norm_weight && !(dims->norm_eps >= 0.0f)) {
        set_error("MoeDims.norm_eps must be >= 0");
        return MOE_ERR_INVALID_ARG;
    }
    return MOE_OK;
}

int enqueue_norm(const MoEArgs* a, const MoeDims* dims, const Shape& s, cudaStream_t stream) {
    if (!dims->norm_weight) return MOE_OK;
    MOE_TRY(launch_rmsnorm(a->input, dims->norm_weight, s, dims->norm_eps, dims->norm_out, stream), "rmsnorm");
    return MOE_OK;
}

// Stages 1-3: router + top-k, slots, gather into the dense expert-major rows.
int enqueue_route(const MoEArgs* a_in, const MoeDims* dims, const Shape& s, const Workspace& ws, cudaStream_t stream) {
    int rc = enqueue_norm(a_in, dims, s, stream);
    if (rc != MOE_OK) return rc;
    const MoEArgs ra = routed_args(a_in, dims);
    const MoEArgs* a = &ra;
    MOE_TRY(launch_router_topk(a->input, a->router_weights, dims->router_bias, s, ws.router_logits, a->expert_logits,
                               a->selected_expert_indices, a->selected_expert_weights, stream),
            "router_topk");
    MOE_TRY(mark_stage(1, stream), "cudaEventRecord(stage event)");
    const FfnBuffers fb = ffn_buffers(a, s);
    MOE_TRY(launch_dispatch_count(a->selected_expert_indices, s, ws, a->expert_counts, nullptr, stream),
            "dispatch (count)");
    MOE_TRY(launch_dispatch_finish(a->input, a->selected_expert_indices, a->selected_expert_weights, s, ws,
                                   scales_of(a, s), dims->slot_base, a->expert_counts, a->expert_token_ids,
                                   a->expert_token_weights, fb.a_rows, stream, dims->skip_gather != 0),
            "dispatch");
    return MOE_OK;
}

// Stage 4: the two grouped GEMMs over the row groups `gt`.
int enqueue_ffn(const MoEArgs* a, const MoeDims* dims, const Shape& s, const GroupTable& gt, int* status,
                float* a_scale, float* h_scale, int num_sms, cudaStream_t stream) {
    const FfnBuffers fb = ffn_buffers(a, s);
    if (s.dtype == MOE_DTYPE_INT4_PTX) {
        // the packed-transposed nibbles are unpacked inside the GEMM (expert_gemm_i4.cu)
        const GemmScales sc = scales_of(a, s);
        MOE_TRY(launch_i4_up_gate(fb.a_rows, fb.wg, fb.wu, s, gt, status, sc, fb.h_rows, stream, num_sms),
                "int4 up/gate GEMM");
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
        MOE_TRY(launch_i4_down(fb.h_rows, fb.wd, s, gt, status, sc, a->hidden_mlp_layer_2_out, stream, num_sms),
                "int4 down GEMM");
        return MOE_OK;
    }
    if (s.dtype == MOE_DTYPE_W4A16) {
        MOE_TRY(launch_w4_up_gate(fb.a_rows, fb.wg, fb.wu, dims->w4_scale_gate, dims->w4_scale_up,
                                  dims->w4_zero_gate, dims->w4_zero_up, s, gt, status, fb.h_rows, stream, num_sms),
                "4-bit up/gate GEMM");
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
        MOE_TRY(launch_w4_down(fb.h_rows, fb.wd, dims->w4_scale_down, dims->w4_zero_down, s, gt, status,
                               a->hidden_mlp_layer_2_out, stream, num_sms),
                "4-bit down GEMM");
        return MOE_OK;
    }
    if (s.dtype == MOE_DTYPE_NVFP4) {
        MOE_TRY(launch_fp4_up_gate(fb.a_rows, fb.wg, fb.wu, dims->w4_scale_gate, dims->w4_scale_up,
                                   dims->fp4_global_gate, dims->fp4_global_up, s, gt, status, fb.h_rows, stream,
                                   num_sms),
                "NVFP4 up/gate GEMM");
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
        MOE_TRY(launch_fp4_down(fb.h_rows, fb.wd, dims->w4_scale_down, dims->fp4_global_down, s, gt, status,
                                a->hidden_mlp_layer_2_out, stream, num_sms),
                "NVFP4 down GEMM");
        return MOE_OK;
    }
    if (s.dtype == MOE_DTYPE_FP8_BLOCK) {
        MOE_TRY(launch_fp8_up_gate(fb.a_rows, a_scale, fb.wg, fb.wu, dims->w_scale_gate, dims->w_scale_up, s, gt,
                                   status, fb.h_rows, h_scale, stream, num_sms),
                "fp8 up/gate GEMM");
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
        MOE_TRY(launch_fp8_down(fb.h_rows, h_scale, fb.wd, dims->w_scale_down, s, gt, status,
                                a->hidden_mlp_layer_2_out, stream, num_sms),
                "fp8 down GEMM");
        return MOE_OK;
    }
    if (s.dtype == MOE_DTYPE_INT8_CHANNEL) {
        MOE_TRY(launch_i8c_up_gate(fb.a_rows, a_scale, fb.wg, fb.wu, dims->w_scale_gate, dims->w_scale_up, s, gt,
                                   status, fb.h_rows, h_scale, stream, num_sms),
                "int8 per-channel up/gate GEMM");
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
        MOE_TRY(launch_i8c_down(fb.h_rows, h_scale, fb.wd, dims->w_scale_down, s, gt, status,
                                a->hidden_mlp_layer_2_out, stream, num_sms),
                "int8 per-channel down GEMM");
        return MOE_OK;
    }
    const GemmScales sc = scales_of(a, s);
    MOE_TRY(launch_expert_up_gate(fb.a_rows, fb.wg, fb.wu, s, gt, status, sc, fb.h_rows, stream, num_sms),
            "expert up/gate GEMM");
    MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
    MOE_TRY(launch_expert_down(fb.h_rows, fb.wd, s, gt, status, sc, a->hidden_mlp_layer_2_out, stream, num_sms),
            "expert down GEMM");
    return MOE_OK;
}

// The stage sequence of one layer call on `stream`, given its scratch.
int enqueue_layer(const MoEArgs* a, const MoeDims* dims, const Shape& s, const Workspace& ws, int num_sms,
                  cudaStream_t stream) {
    MOE_TRY(cudaMemsetAsync(ws.status, 0, sizeof(int), stream), "cudaMemsetAsync(status)");
    MOE_TRY(mark_stage(0, stream), "cudaEventRecord(stage event)");
    int rc = enqueue_route(a, dims, s, ws, stream);
    if (rc != MOE_OK) return rc;
    MOE_TRY(mark_stage(2, stream), "cudaEventRecord(stage event)");
    if (s.T() > 0 && s.cap > 0) {
        const GroupTable gt{ws.expert_rows, ws.expert_start, nullptr, s.E, s.rows_capacity()};
        rc = enqueue_ffn(a, dims, s, gt, ws.status, ws.a_scale, ws.h_scale, num_sms, stream);
        if (rc != MOE_OK) return rc;
    } else {
        MOE_TRY(mark_stage(3, stream), "cudaEventRecord(stage event)");
    }
    MOE_TRY(mark_stage(4, stream), "cudaEventRecord(stage event)");
    MOE_TRY(launch_combine(a->hidden_mlp_layer_2_out, a->selected_expert_indices, a->selected_expert_weights, s, ws,
                           a->final_output, dims->output_16, stream, dims->residual),
            "combine");
    MOE_TRY(mark_stage(5, stream), "cudaEventRecord(stage event)");
    return MOE_OK;
}

}  // namespace moe

extern "C" int moe_solve_v2(const MoEArgs* a, const MoeDims* dims, cudaStream_t stream) {
    Shape s;
    int rc = make_shape(dims, &s);
    if (rc != MOE_OK) return rc;
    rc = check_args(a, s.dtype);
    if (rc != MOE_OK) return rc;
    rc = check_norm(dims);
    if (rc != MOE_OK) return rc;
    DeviceState* st = nullptr;
    int dev = 0;
    rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    rc = resolve_workspace(*st, dev, dims, s, &ws);
    if (rc != MOE_OK) return rc;
    return enqueue_layer(a, dims, s, ws, st->num_sms, stream);
}

// ---- expert-parallel building blocks ---------------------------------------
namespace {
int route_stage_setup(const MoEArgs* a, const MoeDims* dims, const char* who, Shape* s, Workspace* ws) {
    int rc = make_shape(dims, s, /*bind_check=*/false);   // routing needs no weights
    if (rc != MOE_OK) return rc;
    if (!a || !a->input || !a->router_weights || !a->selected_expert_indices || !a->selected_expert_weights ||
        !a->expert_counts || !a->expert_token_ids || !a->expert_token_weights || !ffn_buffers(a, *s).a_rows) {
        set_error("%s: a routing buffer of MoEArgs is null", who);
        return MOE_ERR_INVALID_ARG;
    }
    rc = check_norm(dims);
    if (rc != MOE_OK) return rc;
    DeviceState* st = nullptr;
    int dev = 0;
    rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    return resolve_workspace(*st, dev, dims, *s, ws);
}
}  // namespace

extern "C" int moe_stage_route(const MoEArgs* a, const MoeDims* dims, cudaStream_t stream) {
    Shape s;
    Workspace ws;
    const int rc = route_stage_setup(a, dims, "moe_stage_route", &s, &ws);
    if (rc != MOE_OK) return rc;
    MOE_TRY(cudaMemsetAsync(ws.status, 0, sizeof(int), stream), "cudaMemsetAsync(status)");
    return enqueue_route(a, dims, s, ws, stream);
}

extern "C" int moe_stage_route_counts(const MoEArgs* a, const MoeDims* dims, int* raw_counts, cudaStream_t stream) {
    Shape s;
    Workspace ws;
    const int rc = route_stage_setup(a, dims, "moe_stage_route_counts", &s, &ws);
    if (rc != MOE_OK) return rc;
    if (!raw_counts) { set_error("moe_stage_route_counts: raw_counts is null"); return MOE_ERR_INVALID_ARG; }
    MOE_TRY(cudaMemsetAsync(ws.status, 0, sizeof(int), stream), "cudaMemsetAsync(status)");
    const int nrc = enqueue_norm(a, dims, s, stream);
    if (nrc != MOE_OK) return nrc;
    const MoEArgs ra = routed_args(a, dims);
    MOE_TRY(launch_router_topk(ra.input, a->router_weights, dims->router_bias, s, ws.router_logits, a->expert_logits,
                               a->selected_expert_indices, a->selected_expert_weights, stream),
            "router_topk");
    MOE_TRY(launch_dispatch_count(a->selected_expert_indices, s, ws, a->expert_counts, raw_counts, stream),
            "dispatch (count)");
    return MOE_OK;
}

extern "C" int moe_stage_route_finish(const MoEArgs* a, const MoeDims* dims, cudaStream_t stream) {
    Shape s;
    Workspace ws;
    const int rc = route_stage_setup(a, dims, "moe_stage_route_finish", &s, &ws);
    if (rc != MOE_OK) return rc;
    const FfnBuffers fb = ffn_buffers(a, s);
    MOE_TRY(launch_dispatch_finish(routed_args(a, dims).input, a->selected_expert_indices, a->selected_expert_weights,
                                   s, ws,
                                   scales_of(a, s), dims->slot_base, a->expert_counts, a->expert_token_ids,
                                   a->expert_token_weights, fb.a_rows, stream, dims->skip_gather != 0),
            "dispatch");
    return MOE_OK;
}

namespace {
size_t ffn_h_scale_bytes(const Shape& s, int64_t rows_capacity) {
    if (s.dtype != MOE_DTYPE_FP8_BLOCK && s.dtype != MOE_DTYPE_INT8_CHANNEL) return 0;
    return align256(sizeof(float) * (size_t)rows_capacity * (s.f / 128));
}
}  // namespace

extern "C" size_t moe_ffn_scratch_bytes(const MoeDims* dims, int64_t rows_capacity) {
    if (!dims || rows_capacity < 0 || dims->d_ff <= 0) return 0;
    Shape s;   // only the format and d_ff matter (weights need not be bound yet)
    s.dtype = dims->dtype;
    s.f = dims->d_ff;
    return workspace_header_bytes() + ffn_h_scale_bytes(s, rows_capacity);
}

namespace {
int stage_ffn(const MoEArgs* a, const MoeDims* dims, const int* group_rows, const int* group_start,
              const int* group_expert, const int* group_out_rank, const int* group_out_row, int num_groups,
              int64_t rows_capacity, float* const* out_bases, int num_bases, cudaStream_t stream) {
    // Only the FFN shape matters here: an owner may hold a single expert.
    if (!dims) { set_error("dims is null"); return MOE_ERR_INVALID_ARG; }
    MoeDims fd = *dims;
    fd.num_experts = 8;
    fd.top_k = 1;
    fd.num_batches = 0;
    Shape s;
    int rc = make_shape(&fd, &s);
    if (rc != MOE_OK) return rc;
    s.E = dims->num_experts;
    if (s.E < 1) { set_error("moe_stage_expert_ffn: num_experts %d", s.E); return MOE_ERR_INVALID_ARG; }
    if (!a) { set_error("args is null"); return MOE_ERR_INVALID_ARG; }
    {
        const FfnBuffers fb = ffn_buffers(a, s);
        if (!fb.a_rows || !fb.h_rows || !fb.wg || !fb.wu || !fb.wd || !a->hidden_mlp_layer_2_out) {
            set_error("moe_stage_expert_ffn: a weight or row buffer of MoEArgs is null");
            return MOE_ERR_INVALID_ARG;
        }
    }
    if (!group_rows || !group_start || num_groups < 0 || num_groups > kMaxGroups || rows_capacity < 0 ||
        rows_capacity >= ((int64_t)1 << 31)) {
        set_error("moe_stage_expert_ffn: bad group table (num_groups %d, max %d)", num_groups, kMaxGroups);
        return MOE_ERR_INVALID_ARG;
    }
    if (group_out_rank && (!group_out_row || !out_bases || num_bases < 1 || num_bases > kMaxPeers)) {
        set_error("moe_stage_expert_ffn_peer: out rows / bases missing or more than %d peers", kMaxPeers);
        return MOE_ERR_INVALID_ARG;
    }
    for (int g = 0; g < num_groups; ++g) {
        if (group_out_rank && (group_out_rank[g] < 0 || group_out_rank[g] >= num_bases || group_out_row[g] < 0 ||
                               !out_bases[group_out_rank[g]])) {
            set_error("moe_stage_expert_ffn_peer: group %d has a bad output rank / row", g);
            return MOE_ERR_INVALID_ARG;
        }
        const int w = group_expert ? group_expert[g] : g;
        if (group_rows[g] < 0 || group_start[g] < 0 || (int64_t)group_start[g] + group_rows[g] > rows_capacity ||
            w < 0 || w >= s.E) {
            set_error("moe_stage_expert_ffn: group %d out of range", g);
            return MOE_ERR_INVALID_ARG;
        }
    }
    DeviceState* st = nullptr;
    int dev = 0;
    rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    rc = resolve_workspace(*st, dev, dims, s, &ws, /*header_only=*/true);
    if (rc != MOE_OK) return rc;
    if (num_groups == 0 || rows_capacity == 0) return MOE_OK;
    MOE_TRY(cudaMemcpyAsync(ws.grp_rows, group_rows, sizeof(int) * num_groups, cudaMemcpyHostToDevice, stream),
            "cudaMemcpyAsync(group rows)");
    MOE_TRY(cudaMemcpyAsync(ws.grp_start, group_start, sizeof(int) * num_groups, cudaMemcpyHostToDevice, stream),
            "cudaMemcpyAsync(group starts)");
    if (group_expert)
        MOE_TRY(cudaMemcpyAsync(ws.grp_weight, group_expert, sizeof(int) * num_groups, cudaMemcpyHostToDevice,
                                stream),
                "cudaMemcpyAsync(group experts)");
    GroupTable gt{ws.grp_rows, ws.grp_start, group_expert ? ws.grp_weight : nullptr, num_groups, rows_capacity};
    if (group_out_rank) {
        MOE_TRY(cudaMemcpyAsync(ws.grp_out_rank, group_out_rank, sizeof(int) * num_groups, cudaMemcpyHostToDevice,
                                stream),
                "cudaMemcpyAsync(group output ranks)");
        MOE_TRY(cudaMemcpyAsync(ws.grp_out_row, group_out_row, sizeof(int) * num_groups, cudaMemcpyHostToDevice,
                                stream),
                "cudaMemcpyAsync(group output rows)");
        gt.redirect.rank = ws.grp_out_rank;
        gt.redirect.row0 = ws.grp_out_row;
        for (int r = 0; r < num_bases; ++r) gt.redirect.bases[r] = out_bases[r];
    }
    float* h_scale = nullptr;
    if (s.dtype == MOE_DTYPE_FP8_BLOCK || s.dtype == MOE_DTYPE_INT8_CHANNEL) {
        // row scales of A from the caller; h scales in the caller's scratch after the header
        if (!dims->act_scale || !dims->scratch ||
            dims->scratch_bytes < workspace_header_bytes() + ffn_h_scale_bytes(s, rows_capacity)) {
            set_error("moe_stage_expert_ffn: FP8_BLOCK / INT8_CHANNEL need MoeDims.act_scale and a scratch of "
                      "moe_ffn_scratch_bytes()");
            return MOE_ERR_INVALID_ARG;
        }
        h_scale = reinterpret_cast<float*>(static_cast<uint8_t*>(dims->scratch) + workspace_header_bytes());
    }
    return enqueue_ffn(a, dims, s, gt, ws.status, dims->act_scale, h_scale, st->num_sms, stream);
}
}  // namespace

extern "C" int moe_stage_expert_ffn(const MoEArgs* a, const MoeDims* dims, const int* group_rows,
                                    const int* group_start, const int* group_expert, int num_groups,
                                    int64_t rows_capacity, cudaStream_t stream) {
    return stage_ffn(a, dims, group_rows, group_start, group_expert, nullptr, nullptr, num_groups, rows_capacity,
                     nullptr, 0, stream);
}

extern "C" int moe_stage_expert_ffn_peer(const MoEArgs* a, const MoeDims* dims, const int* group_rows,
                                         const int* group_start, const int* group_expert, const int* group_out_rank,
                                         const int* group_out_row, int num_groups, int64_t rows_capacity,
                                         float* const* out_bases, int num_bases, cudaStream_t stream) {
    if (!group_out_rank) { set_error("moe_stage_expert_ffn_peer: group_out_rank is null"); return MOE_ERR_INVALID_ARG; }
    return stage_ffn(a, dims, group_rows, group_start, group_expert, group_out_rank, group_out_row, num_groups,
                     rows_capacity, out_bases, num_bases, stream);
}

extern "C" int moe_ep_plan(const int* table, int world, int rank, int num_experts, int strided, int* plan,
                           cudaStream_t stream) {
    if (!table || !plan || world < 1 || world > kMaxPeers || rank < 0 || rank >= world || num_experts < 1 ||
        num_experts % world != 0 || num_experts > kMaxGroups) {
        set_error("moe_ep_plan: bad arguments (world %d, rank %d, experts %d)", world, rank, num_experts);
        return MOE_ERR_INVALID_ARG;
    }
    MOE_TRY(launch_ep_plan(table, world, num_experts, rank, strided != 0, plan, stream), "ep plan");
    return MOE_OK;
}

extern "C" int moe_stage_dispatch_peer(const MoEArgs* a, const MoeDims* dims, const int* plan,
                                       void* const* row_bases, float* const* scale_bases, int num_bases,
                                       cudaStream_t stream) {
    Shape s;
    Workspace ws;
    const int rc = route_stage_setup(a, dims, "moe_stage_dispatch_peer", &s, &ws);
    if (rc != MOE_OK) return rc;
    const bool scaled = s.dtype == MOE_DTYPE_FP8_BLOCK || s.dtype == MOE_DTYPE_INT8_CHANNEL;
    if (!plan || !row_bases || num_bases < 1 || num_bases > kMaxPeers || (scaled && !scale_bases)) {
        set_error("moe_stage_dispatch_peer: plan / bases missing or more than %d peers", kMaxPeers);
        return MOE_ERR_INVALID_ARG;
    }
    GatherDst gd;
    for (int r = 0; r < num_bases; ++r) {
        gd.rows[r] = row_bases[r];
        gd.scales[r] = scaled ? scale_bases[r] : nullptr;
    }
    gd.rank = plan;
    gd.row0 = plan + s.E;
    MOE_TRY(launch_dispatch_gather(routed_args(a, dims).input, a->selected_expert_indices, s, ws, scales_of(a, s), gd,
                                   stream),
            "dispatch (peer gather)");
    return MOE_OK;
}

extern "C" int moe_stage_expert_ffn_planned(const MoEArgs* a, const MoeDims* dims, const int* plan, int num_groups,
                                            int64_t rows_capacity, float* const* out_bases, int num_bases,
                                            cudaStream_t stream) {
    if (!dims || !a || !plan || !out_bases || num_bases < 1 || num_bases > kMaxPeers || num_groups < 0 ||
        num_groups > kMaxGroups || rows_capacity < 0 || rows_capacity >= ((int64_t)1 << 31)) {
        set_error("moe_stage_expert_ffn_planned: bad arguments");
        return MOE_ERR_INVALID_ARG;
    }
    MoeDims fd = *dims;
    fd.num_experts = 8;
    fd.top_k = 1;
    fd.num_batches = 0;
    Shape s;
    int rc = make_shape(&fd, &s);
    if (rc != MOE_OK) return rc;
    s.E = dims->num_experts;
    const FfnBuffers fb = ffn_buffers(a, s);
    if (!fb.a_rows || !fb.h_rows || !fb.wg || !fb.wu || !fb.wd || !a->hidden_mlp_layer_2_out) {
        set_error("moe_stage_expert_ffn_planned: a weight or row buffer of MoEArgs is null");
        return MOE_ERR_INVALID_ARG;
    }
    DeviceState* st = nullptr;
    int dev = 0;
    rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    rc = resolve_workspace(*st, dev, dims, s, &ws, /*header_only=*/true);
    if (rc != MOE_OK) return rc;
    if (num_groups == 0 || rows_capacity == 0) return MOE_OK;
    const int E = num_groups;   // plan arrays are E long
    GroupTable gt{plan + 2 * E, plan + 3 * E, plan + 4 * E, num_groups, rows_capacity};
    gt.redirect.rank = plan + 5 * E;
    gt.redirect.row0 = plan + 6 * E;
    for (int r = 0; r < num_bases; ++r) gt.redirect.bases[r] = out_bases[r];
    float* h_scale = nullptr;
    if (s.dtype == MOE_DTYPE_FP8_BLOCK || s.dtype == MOE_DTYPE_INT8_CHANNEL) {
        if (!dims->act_scale || !dims->scratch ||
            dims->scratch_bytes < workspace_header_bytes() + ffn_h_scale_bytes(s, rows_capacity)) {
            set_error("moe_stage_expert_ffn_planned: FP8_BLOCK / INT8_CHANNEL need MoeDims.act_scale and a scratch "
                      "of moe_ffn_scratch_bytes()");
            return MOE_ERR_INVALID_ARG;
        }
        h_scale = reinterpret_cast<float*>(static_cast<uint8_t*>(dims->scratch) + workspace_header_bytes());
    }
    return enqueue_ffn(a, dims, s, gt, ws.status, dims->act_scale, h_scale, st->num_sms, stream);
}

extern "C" int moe_stage_combine(const MoEArgs* a, const MoeDims* dims, cudaStream_t stream) {
    Shape s;
    int rc = make_shape(dims, &s, /*bind_check=*/false);
    if (rc != MOE_OK) return rc;
    if (!a || !a->hidden_mlp_layer_2_out || !a->final_output || !a->selected_expert_indices ||
        !a->selected_expert_weights) {
        set_error("moe_stage_combine: null buffer");
        return MOE_ERR_INVALID_ARG;
    }
    DeviceState* st = nullptr;
    int dev = 0;
    rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    if (dims->scratch) {
        rc = resolve_workspace(*st, dev, dims, s, &ws);
        if (rc != MOE_OK) return rc;
    } else {
        std::lock_guard<std::mutex> lk(g_mu);
        if (st->ws_bytes < workspace_bytes(s)) {
            set_error("moe_stage_combine: no routing tables for these dims (run moe_stage_route first)");
            return MOE_ERR_INVALID_ARG;
        }
        carve_workspace(st->ws, s, &ws);
    }
    MOE_TRY(launch_combine(a->hidden_mlp_layer_2_out, a->selected_expert_indices, a->selected_expert_weights, s, ws,
                           a->final_output, dims->output_16, stream, dims->residual),
            "combine");
    return MOE_OK;
}

extern "C" int moe_set_stage_events(void* const* events, int count) {
    if (count == 0) { g_stage_on = false; return MOE_OK; }
    if (!events || count != kStageEvents) {
        set_error("moe_set_stage_events needs %d events (or count 0)", kStageEvents);
        return MOE_ERR_INVALID_ARG;
    }
    for (int i = 0; i < kStageEvents; ++i) g_stage_ev[i] = static_cast<cudaEvent_t>(events[i]);
    g_stage_on = true;
    return MOE_OK;
}

extern "C" int moe_check_device_status(cudaStream_t stream) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev >= kMaxDevices || !g_dev[dev].status) return MOE_OK;
    int host = 0;
    e = cudaMemcpy(&host, g_dev[dev].status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
    if (host != 0) {
        set_error("device-side wait timed out (status %d)", host);
        return MOE_ERR_TIMEOUT;
    }
    return MOE_OK;
}

extern "C" int moe_selftest_wait_timeout(int64_t timeout_ns, cudaStream_t stream) {
    if (timeout_ns <= 0 || timeout_ns > 10000000000ll) {
        set_error("timeout_ns must be in (0, 10 s]");
        return MOE_ERR_INVALID_ARG;
    }
    DeviceState* st = nullptr;
    int dev = 0;
    int rc = device_state(&st, &dev);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        rc = get_workspace(*st, Shape{}, &ws, /*header_only=*/true);
    }
    if (rc != MOE_OK) return rc;
    MOE_TRY(cudaMemsetAsync(ws.status, 0, sizeof(int), stream), "cudaMemsetAsync(status)");
    MOE_TRY(launch_wait_selftest(ws.status, (uint64_t)timeout_ns, stream), "wait self-test");
    note_status_word(dev, ws.status);
    return MOE_OK;
}

extern "C" void moe_release(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return;
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& st = g_dev[dev];
    if (st.ws) cudaFree(st.ws);
    st.ws = nullptr;
    st.ws_bytes = 0;
    st.status = nullptr;
}

// kernels/launcher.h:21-48: launch, synchronise, time with events, print the
// duration line, exit(1) on any error.
extern "C" void solve(MoEArgs args) {
    MoeDims dims;
    moe_get_solve_dims(&dims);
    dims.num_batches = args.num_batches;
    dims.cap = args.use_capacity ? (args.cap > 0 ? args.cap : 0) : -1;
    auto die = [](const char* what) {
        fprintf(stderr, "CUDA Error at: %s: %s \n", what, moe_last_error());
        exit(1);
    };
    // The reference picks the kernel at build time (Makefile KERNEL=) and the
    // allocator at run time (drivers/main.cu:84-106); here the weight fields
    // that allocator filled in pick the path: fp16 -> capacity, int4 (its
    // int4_ptx allocator also fills the int8 fields) -> capacity_int4_ptx,
    // int8 alone -> capacity_int8_ptx, fp8 -> capacity_fp8_ptx.
    const bool per_tensor = dims.dtype == MOE_DTYPE_INT8 || dims.dtype == MOE_DTYPE_INT4_PTX ||
                            dims.dtype == MOE_DTYPE_FP8;
    if (args.expert_up_proj_weights) {
        if (per_tensor) dims.dtype = MOE_DTYPE_F16;
    } else if (args.expert_up_proj_weights_int4) {
        dims.dtype = MOE_DTYPE_INT4_PTX;
    } else if (args.expert_up_proj_weights_int8) {
        dims.dtype = MOE_DTYPE_INT8;
    } else if (args.expert_up_proj_weights_fp8) {
        dims.dtype = MOE_DTYPE_FP8;
    } else {
        set_error("solve(): no expert weights in MoEArgs");
        die("solve");
    }
    cudaEvent_t start, stop;
    if (cudaEventCreate(&start) != cudaSuccess || cudaEventCreate(&stop) != cudaSuccess) {
        set_error("cudaEventCreate failed");
        die("solve");
    }
    cudaEventRecord(start);
    if (moe_solve_v2(&args, &dims, 0) != MOE_OK) die("moe_solve_v2");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { set_error("%s", cudaGetErrorString(e)); die("cudaDeviceSynchronize"); }
    if (moe_check_device_status(0) != MOE_OK) die("moe_check_device_status");
    cudaEventRecord(stop);
    cudaEventSynchronize(stop);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, start, stop);
    printf("Total duration via cudaEventRecord: %.3f ms\n", ms);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
}
