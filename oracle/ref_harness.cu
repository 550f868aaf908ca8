// Golden-vector harness (test infrastructure): runs the reference's
// multi-launch path (kernels/unfused.cu `solve`, the only reference GPU path
// whose stages are separated by kernel boundaries) on inputs read from files
// and writes its routing tables and output back.  Built against the shadow
// config in oracle/ref_shadow by oracle/build_ref.sh.
//
//   ref_unfused <in_dir> <out_dir>
//   in:  x.bin [B,N,d] f16, wr.bin [d,E] f16, wg.bin / wu.bin [E,d,f] f16, wd.bin [E,f,d] f16
//   out: logits.bin [B,N,E] f32, idx.bin [B,N,k] i32, w.bin [B,N,k] f32,
//        counts.bin [B,E] i32, out.bin [B,N,d] f32
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include "include/config.h"
#include "include/moe_args.h"

extern "C" void solve(MoEArgs args);

#define HCHECK(x)                                                                        \
    do {                                                                                 \
        cudaError_t e_ = (x);                                                            \
        if (e_ != cudaSuccess) {                                                         \
            fprintf(stderr, "harness: %s failed: %s\n", #x, cudaGetErrorString(e_));    \
            exit(2);                                                                     \
        }                                                                                \
    } while (0)

static std::vector<char> read_file(const std::string& p, size_t bytes) {
    std::vector<char> b(bytes);
    FILE* f = fopen(p.c_str(), "rb");
    if (!f || fread(b.data(), 1, bytes, f) != bytes) {
        fprintf(stderr, "harness: cannot read %zu bytes from %s\n", bytes, p.c_str());
        exit(2);
    }
    fclose(f);
    return b;
}
static void write_file(const std::string& p, const void* d, size_t bytes) {
    FILE* f = fopen(p.c_str(), "wb");
    if (!f || fwrite(d, 1, bytes, f) != bytes) {
        fprintf(stderr, "harness: cannot write %s\n", p.c_str());
        exit(2);
    }
    fclose(f);
}
template <class T>
static T* dev_upload(const std::vector<char>& h) {
    T* d = nullptr;
    HCHECK(cudaMalloc(&d, h.size()));
    HCHECK(cudaMemcpy(d, h.data(), h.size(), cudaMemcpyHostToDevice));
    return d;
}
template <class T>
static T* dev_alloc(size_t n) {
    T* d = nullptr;
    HCHECK(cudaMalloc(&d, n * sizeof(T)));
    HCHECK(cudaMemset(d, 0, n * sizeof(T)));
    return d;
}
template <class T>
static std::vector<T> download(const T* d, size_t n) {
    std::vector<T> h(n);
    HCHECK(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost));
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
    MoEArgs a{};
    a.num_batches = (int)B;
    a.use_capacity = false;
    a.cap = (int)Nt;
    a.input = dev_upload<half>(read_file(in + "/x.bin", B * Nt * d * 2));
    a.router_weights = dev_upload<half>(read_file(in + "/wr.bin", d * E * 2));
    a.expert_gate_proj_weights = dev_upload<half>(read_file(in + "/wg.bin", E * d * f * 2));
    a.expert_up_proj_weights = dev_upload<half>(read_file(in + "/wu.bin", E * d * f * 2));
    a.expert_down_proj_weights = dev_upload<half>(read_file(in + "/wd.bin", E * f * d * 2));
    const size_t rows = B * E * Nt;
    a.expert_logits = dev_alloc<float>(B * Nt * E);
    a.selected_expert_indices = dev_alloc<int>(B * Nt * kk);
    a.selected_expert_weights = dev_alloc<float>(B * Nt * kk);
    a.expert_counts = dev_alloc<int>(B * E);
    a.expert_token_ids = dev_alloc<int>(rows);
    a.expert_token_weights = dev_alloc<float>(rows);
    a.per_expert_wmma_inputs = dev_alloc<half>(rows * d);
    a.hidden_mlp_layer_1_out = dev_alloc<float>(rows * f);
    a.hidden_mlp_gate_out = dev_alloc<float>(rows * f);
    a.hidden_mlp_layer_1_out_fp16 = dev_alloc<half>(rows * f);
    a.hidden_mlp_layer_2_out = dev_alloc<float>(rows * d);
    a.final_output = dev_alloc<float>(B * Nt * d);
    solve(a);
    HCHECK(cudaDeviceSynchronize());
    auto lg = download(a.expert_logits, B * Nt * E);
    auto ix = download(a.selected_expert_indices, B * Nt * kk);
    auto w = download(a.selected_expert_weights, B * Nt * kk);
    auto c = download(a.expert_counts, B * E);
    auto o = download(a.final_output, B * Nt * d);
    write_file(out + "/logits.bin", lg.data(), lg.size() * 4);
    write_file(out + "/idx.bin", ix.data(), ix.size() * 4);
    write_file(out + "/w.bin", w.data(), w.size() * 4);
    write_file(out + "/counts.bin", c.data(), c.size() * 4);
    write_file(out + "/out.bin", o.data(), o.size() * 4);
    printf("harness ok: B=%zu N=%zu d=%zu f=%zu E=%zu k=%zu\n", B, Nt, d, f, E, kk);
    return 0;
}
