// Pin harness (test infrastructure): runs one of the reference's fused kernels
// (kernels/capacity.cu, capacity_int8_ptx.cu, capacity_int4_ptx.cu or
// capacity_fp8_ptx.cu, compiled in beside this file against the shadow
// config in oracle/ref_shadow) once on inputs read from files, and writes the
// routing tables and output back, so that the oracle's restatement of that
// kernel's arithmetic can be checked against the kernel itself.
//
// The fused kernels separate their stages with __syncthreads() only, route
// tokens from blockIdx.x alone and cover a partial grid of rows, so they
// compute their intended semantics only when the whole problem fits one
// thread block: the builder (oracle/build_ref_kernels.sh) uses N = 16, d = f
// = 64, one batch, so gridDim = (1, 1, 1); the 8 tokens the block routes are
// the ones compared.  Routing tables start at -1 / 0 so that tokens the block
// does not route take no capacity slots.
//
//   ref_pin_<kernel> <in_dir> <out_dir>
//   in:  x.bin [B,N,d] f16, wr.bin [d,E] f16, scales.bin 5 x f32 (s_up, s_gate,
//        s_down, s_in, s_mid), and per matrix (wg / wu / wd) one of
//        <m>.bin f16, <m>_i8.bin int8, <m>_i4.bin packed-transposed int4,
//        <m>_f8.bin e4m3 codes
//   out: idx.bin [B,N,k] i32, counts.bin [B,E] i32, token_ids.bin
//        [B,E,CAP] i32, out.bin [B,N,d] f32
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include "include/config.h"
#include "include/moe_args.h"

extern "C" void solve(MoEArgs args);

#define PCHECK(x)                                                                        \
    do {                                                                                 \
        cudaError_t e_ = (x);                                                            \
        if (e_ != cudaSuccess) {                                                         \
            fprintf(stderr, "ref_pin: %s failed: %s\n", #x, cudaGetErrorString(e_));    \
            exit(2);                                                                     \
        }                                                                                \
    } while (0)

static bool read_file(const std::string& p, std::vector<char>& b, size_t bytes) {
    FILE* f = fopen(p.c_str(), "rb");
    if (!f) return false;
    b.resize(bytes);
    const bool ok = fread(b.data(), 1, bytes, f) == bytes;
    fclose(f);
    if (!ok) {
        fprintf(stderr, "ref_pin: short read of %s\n", p.c_str());
        exit(2);
    }
    return true;
}
static void write_file(const std::string& p, const void* d, size_t bytes) {
    FILE* f = fopen(p.c_str(), "wb");
    if (!f || fwrite(d, 1, bytes, f) != bytes) {
        fprintf(stderr, "ref_pin: cannot write %s\n", p.c_str());
        exit(2);
    }
    fclose(f);
}
template <class T>
static T* upload(const std::vector<char>& h) {
    void* d = nullptr;
    PCHECK(cudaMalloc(&d, h.size()));
    PCHECK(cudaMemcpy(d, h.data(), h.size(), cudaMemcpyHostToDevice));
    return static_cast<T*>(d);
}
template <class T>
static T* zeros(size_t n, int byte = 0) {
    void* d = nullptr;
    PCHECK(cudaMalloc(&d, n * sizeof(T) + 256));
    PCHECK(cudaMemset(d, byte, n * sizeof(T) + 256));
    return static_cast<T*>(d);
}
template <class T>
static std::vector<T> download(const T* d, size_t n) {
    std::vector<T> h(n);
    PCHECK(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost));
    return h;
}

int main(int argc, char** argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s <in_dir> <out_dir>\n", argv[0]);
        return 2;
    }
    const std::string in = argv[1], out = argv[2];
    const size_t B = num_batches, Nt = N, d = d_model, f = (size_t)up_proj_dim * d_model, E = num_experts,
                 kk = k;
    // CAP as the fused kernels compute it (e.g. kernels/capacity.cu:502-503)
    const int cap_raw = (int)ceilf((float)N * (float)k / (float)num_experts * capacity_factor);
    const size_t CAP = (size_t)(((cap_raw + WMMA_M - 1) / WMMA_M) * WMMA_M);
    const size_t rows = B * E * CAP;
    MoEArgs a{};
    a.num_batches = (int)B;
    a.use_capacity = true;
    a.cap = (int)CAP;
    std::vector<char> buf;
    if (!read_file(in + "/x.bin", buf, B * Nt * d * 2)) {
        fprintf(stderr, "ref_pin: x.bin missing\n");
        return 2;
    }
    a.input = upload<half>(buf);
    if (read_file(in + "/wr.bin", buf, d * E * 2)) a.router_weights = upload<half>(buf);
    struct M { const char* name; size_t K, Nc; const half** f16; const int8_t** i8; const uint8_t** i4;
               const __nv_fp8_e4m3** f8; };
    const M mats[3] = {
        {"wg", d, f, &a.expert_gate_proj_weights, &a.expert_gate_proj_weights_int8,
         &a.expert_gate_proj_weights_int4, &a.expert_gate_proj_weights_fp8},
        {"wu", d, f, &a.expert_up_proj_weights, &a.expert_up_proj_weights_int8, &a.expert_up_proj_weights_int4,
         &a.expert_up_proj_weights_fp8},
        {"wd", f, d, &a.expert_down_proj_weights, &a.expert_down_proj_weights_int8,
         &a.expert_down_proj_weights_int4, &a.expert_down_proj_weights_fp8}};
    for (const M& m : mats) {
        const size_t n = E * m.K * m.Nc;
        const std::string base = in + "/" + m.name;
        if (read_file(base + ".bin", buf, n * 2)) *m.f16 = upload<half>(buf);
        if (read_file(base + "_i8.bin", buf, n)) *m.i8 = upload<int8_t>(buf);
        if (read_file(base + "_i4.bin", buf, n / 2)) *m.i4 = upload<uint8_t>(buf);
        if (read_file(base + "_f8.bin", buf, n)) *m.f8 = upload<__nv_fp8_e4m3>(buf);
    }
    if (read_file(in + "/scales.bin", buf, 5 * sizeof(float))) {
        const float* s = reinterpret_cast<const float*>(buf.data());
        a.scale_up_w = s[0];
        a.scale_gate_w = s[1];
        a.scale_down_w = s[2];
        a.scale_input_act = s[3];
        a.scale_mid_act = s[4];
    }
    a.expert_logits = zeros<float>(B * Nt * E);
    a.selected_expert_indices = zeros<int>(B * Nt * kk, 0xFF);   // -1: not routed
    a.selected_expert_weights = zeros<float>(B * Nt * kk);
    a.expert_counts = zeros<int>(B * E);
    a.expert_token_ids = zeros<int>(rows, 0xFF);
    a.expert_token_weights = zeros<float>(rows);
    a.per_expert_wmma_inputs = zeros<half>(rows * d);
    a.per_expert_wmma_inputs_int8 = zeros<int8_t>(rows * d);
    a.per_expert_wmma_inputs_int4 = zeros<uint8_t>(rows * d / 2);
    a.per_expert_wmma_inputs_fp8 = zeros<__nv_fp8_e4m3>(rows * d);
    a.hidden_mlp_layer_1_out = zeros<float>(rows * f);
    a.hidden_mlp_gate_out = zeros<float>(rows * f);
    a.hidden_mlp_layer_1_out_fp16 = zeros<half>(rows * f);
    a.hidden_mlp_layer_1_out_int8 = zeros<int8_t>(rows * f);
    a.hidden_mlp_layer_1_out_int4 = zeros<uint8_t>(rows * f / 2);
    a.hidden_mlp_layer_1_out_fp8 = zeros<__nv_fp8_e4m3>(rows * f);
    a.hidden_mlp_layer_2_out = zeros<float>(rows * d);
    a.final_output = zeros<float>(B * Nt * d);
    solve(a);
    PCHECK(cudaDeviceSynchronize());
    auto ix = download(a.selected_expert_indices, B * Nt * kk);
    auto c = download(a.expert_counts, B * E);
    auto ti = download(a.expert_token_ids, rows);
    auto o = download(a.final_output, B * Nt * d);
    write_file(out + "/idx.bin", ix.data(), ix.size() * 4);
    write_file(out + "/counts.bin", c.data(), c.size() * 4);
    write_file(out + "/token_ids.bin", ti.data(), ti.size() * 4);
    write_file(out + "/out.bin", o.data(), o.size() * 4);
    printf("ref_pin ok: B=%zu N=%zu d=%zu f=%zu E=%zu k=%zu CAP=%zu\n", B, Nt, d, f, E, kk, CAP);
    return 0;
}
