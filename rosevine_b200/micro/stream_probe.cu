// stream_probe.cu - how fast one SM streams weights from HBM while every SM does (sm_100a).
//
// The decode kernels stream expert weight rows into shared-memory rings with 1-D bulk copies
// (cp.async.bulk), a few large copies per ring slot. This program measures whether that form
// limits them: each CTA (one per SM) streams its own 4.5 MB range, 48 KB at a time, either
// through a ring of 2 or 4 shared-memory slots filled by bulk copies (each slot's 48 KB split
// into 1, 4, 16 or 32 copies issued by as many threads) or through registers (16-byte loads, 2,
// 4 or 8 in flight per thread). Inputs exceed L2 and an L2-sized buffer is rewritten before each
// timed launch; the best of 4 launches after one warm-up, timed with CUDA events.
//
// Build and run (on a B200, from this directory):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o stream_probe stream_probe.cu
//   ./stream_probe          (one JSON line per configuration; about 2 s)
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "../csrc/common.cuh"
using namespace rvc;

constexpr int CHUNK = 48 * 1024;
constexpr int NCHUNK = 96;  // per CTA
constexpr size_t PER_CTA = (size_t)CHUNK * NCHUNK;

__global__ void __launch_bounds__(512, 1) k_bulk(const uint8_t *src, int nslot, int parts, unsigned *err, unsigned *sink) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[8];
    const int tid = threadIdx.x;
    const uint8_t *base = src + (size_t)blockIdx.x * PER_CTA;
    const uint32_t part = CHUNK / parts;
    if (tid == 0) {
        for (int s = 0; s < nslot; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int k) {  // threads < parts
        const int s = k % nslot;
        if (tid == 0) mbar_arrive_expect_tx(&full[s], CHUNK);
        if (tid < parts) bulk_g2s(smem + (size_t)s * CHUNK + tid * part, base + (size_t)k * CHUNK + tid * part, part, &full[s]);
    };
    for (int k = 0; k < nslot && k < NCHUNK; ++k) issue(k);
    unsigned acc = 0;
    bool bad = false;
    int k = 0;
    for (; k < NCHUNK; ++k) {
        const int s = k % nslot;
        bool ok = false;
        for (int i = 0; i < (1 << 22) && !ok; ++i) ok = mbar_try_wait(&full[s], (uint32_t)(k / nslot) & 1u);
        if (__syncthreads_or(!ok)) { bad = true; break; }
        acc += reinterpret_cast<const unsigned *>(smem + (size_t)s * CHUNK)[tid];
        __syncthreads();
        if (k + nslot < NCHUNK) issue(k + nslot);
    }
    if (bad && tid == 0) {
        atomicAdd(err, 1u);
        for (int j = k; j < NCHUNK && j < k + nslot; ++j)  // drain what is in flight (bounded)
            for (int i = 0; i < (1 << 22) && !mbar_try_wait(&full[j % nslot], (uint32_t)(j / nslot) & 1u); ++i) {
            }
    }
    if (acc == 0x12345678u) sink[0] = acc;
}

template <int U>
__global__ void __launch_bounds__(512, 1) k_ldg(const uint8_t *src, unsigned *sink) {
    const uint4 *p = reinterpret_cast<const uint4 *>(src + (size_t)blockIdx.x * PER_CTA);
    const int n = PER_CTA / 16;
    unsigned acc = 0;
    for (int i = threadIdx.x; i < n; i += 512 * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = i + u * 512;
            v[u] = j < n ? __ldcs(p + j) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) acc += v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    if (acc == 0x12345678u) sink[0] = acc;
}

int main() {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const size_t total = PER_CTA * sms;
    uint8_t *src;
    unsigned *err, *sink;
    uint8_t *flush;
    cudaMalloc(&src, total);
    cudaMalloc(&flush, 256 << 20);
    cudaMalloc(&err, 4);
    cudaMalloc(&sink, 4);
    cudaMemset(src, 1, total);
    cudaMemset(err, 0, 4);
    cudaFuncSetAttribute(k_bulk, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * CHUNK);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    auto run = [&](const char *name, auto launch) {
        float best = 1e9f;
        for (int r = 0; r < 5; ++r) {
            cudaMemsetAsync(flush, r, 256 << 20);
            cudaEventRecord(a);
            launch();
            cudaEventRecord(b);
            cudaEventSynchronize(b);
            float ms;
            cudaEventElapsedTime(&ms, a, b);
            if (r > 0 && ms < best) best = ms;
        }
        unsigned e = 0;
        cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost);
        printf("{\"probe\": \"%s\", \"us\": %.1f, \"GBps\": %.0f, \"per_sm_Bpc\": %.2f, \"err\": %u, \"cuda\": \"%s\"}\n", name,
               best * 1e3, total / (best * 1e-3) / 1e9, total / (double)sms / (best * 1e-3) / 1.965e9, e,
               cudaGetErrorString(cudaGetLastError()));
    };
    for (int nslot : {2, 4})
        for (int parts : {1, 4, 16, 32}) {
            char nm[64];
            snprintf(nm, 64, "bulk slots=%d parts=%d", nslot, parts);
            run(nm, [&] { k_bulk<<<sms, 512, nslot * CHUNK>>>(src, nslot, parts, err, sink); });
        }
    run("ldg u=2", [&] { k_ldg<2><<<sms, 512>>>(src, sink); });
    run("ldg u=4", [&] { k_ldg<4><<<sms, 512>>>(src, sink); });
    run("ldg u=8", [&] { k_ldg<8><<<sms, 512>>>(src, sink); });
    return 0;
}
