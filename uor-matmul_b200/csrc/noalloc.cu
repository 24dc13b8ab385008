// noalloc.cu -- the exact i8 GEMM for callers that cannot allocate device memory.
//
// Same kernels as the context path (K1 in chunk mode, then the exact chunk fold),
// but every byte of working memory comes from one file-scope device array, so the
// call makes no cudaMalloc/cudaFree and calls no allocating library routine.
#include <climits>
#include <mutex>
#include "internal.h"
#include "aux.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

using namespace uor;

// Layout: [0, 256) the bounded-wait status word; [256, end) s32 chunk partials.
static __device__ __align__(256) unsigned char g_noalloc_scratch[UOR_B200_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kStatusBytes = 256;

// The array's device address, looked up once per device with that device current.
// In host code the symbol is only a host-side stand-in; this is the usable address.
unsigned char* scratch_address(int* status) {
    static unsigned char* addr[64] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        *status = UOR_B200_DEVICE_ERROR;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            *status = UOR_B200_DEVICE_ERROR;
            return nullptr;
        }
        addr[dev] = static_cast<unsigned char*>(p);
    }
    return addr[dev];
}

bool tma_readable(const void* p, size_t rows, size_t ld) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (rows <= 1 || (ld % 16) == 0);
}

}  // namespace

extern "C" int uor_b200_gemm_ex_i8_noalloc(uor_b200_dtype out, size_t m, size_t k, size_t n,
                                           int64_t alpha, const int8_t* a, size_t lda,
                                           const int8_t* b, size_t ldb, int64_t beta, void* c,
                                           size_t ldc, uint32_t encode, void* stream_ptr) {
    int kind;
    switch (out) {
    case UOR_B200_I8: kind = OUT_I8; break;
    case UOR_B200_I16: kind = OUT_I16; break;
    case UOR_B200_I32: kind = OUT_I32; break;
    case UOR_B200_I64: kind = OUT_I64; break;
    case UOR_B200_I128: kind = OUT_I128; break;
    default: return UOR_B200_UNSUPPORTED;
    }
    if (encode > 3) return UOR_B200_INVALID_ARGUMENT;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if ((m > 1 && ldc < n) || (k && (lda < k || ldb < n))) return UOR_B200_INVALID_ARGUMENT;
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    const bool chunked = (int64_t)k > K1_LANE_DEPTH;
    const size_t chunks = chunked ? (k + K1_CHUNK_K - 1) / K1_CHUNK_K : 1;
    if (chunked) {
        // chunks * m * n s32 partials must fit; compared by division, so no product of
        // the three sizes is formed (it could wrap size_t before the comparison).
        const size_t cells = (UOR_B200_NOALLOC_SCRATCH_BYTES - kStatusBytes) / sizeof(int32_t);
        if (m > cells / n || m * n > cells / chunks) return UOR_B200_SCRATCH_LIMIT;
    }
    if (k && (!tma_readable(a, m, lda) || !tma_readable(b, k, ldb))) return UOR_B200_UNSUPPORTED;

    int st = UOR_B200_OK;
    unsigned char* scratch = scratch_address(&st);
    if (!scratch) return st;
    int* status = reinterpret_cast<int*>(scratch);
    int32_t* part = reinterpret_cast<int32_t*>(scratch + kStatusBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // The status word must start at zero; the partials are fully overwritten.
    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;

    const LinearEpi epi{alpha, beta, (int)encode, kind};
    cudaError_t e = cudaSuccess;
    if (k == 0) {
        e = epilogue_only(c, (int64_t)ldc, 1, m, n, epi, s);
    } else {
        CUtensorMap tmA, tmB;
        const uint64_t sa = m <= 1 ? (k + 15) / 16 * 16 : lda;
        const uint64_t sb = k <= 1 ? (n + 15) / 16 * 16 : ldb;
        if (!make_tmap_u8(&tmA, a, k, m, sa, 128, 128) || !make_tmap_u8(&tmB, b, n, k, sb, 128, 128))
            return UOR_B200_DEVICE_ERROR;
        K1Params p{};
        p.m = (int)m;
        p.n = (int)n;
        p.tiles_m = (int)((m + K1_BM - 1) / K1_BM);
        p.tiles_n = (int)((n + K1_BN - 1) / K1_BN);
        p.num_tiles = p.tiles_m * p.tiles_n;
        p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
        p.idesc = idesc_i8(K1_BM, K1_BN, true, true, false, true);
        p.status = status;
        p.budget_ns = 2000000000ull;
        const int grid = p.num_tiles < sms ? p.num_tiles : sms;
        if (!chunked) {
            p.num_kb = (int)((k + K1_BK - 1) / K1_BK);
            p.c = c;
            p.rsc = (int64_t)ldc;
            p.csc = 1;
            p.epi = epi;
            p.fast = kind == OUT_I32 && alpha == 1 && beta == 0 &&
                     (m == 1 || (ldc % 4) == 0) && (reinterpret_cast<uintptr_t>(c) & 15u) == 0;
            e = k1_launch(tmA, tmB, false, true, p, grid, s);
        } else {
            for (size_t q = 0; q < chunks && e == cudaSuccess; ++q) {
                const size_t k0 = q * K1_CHUNK_K;
                const size_t kl = (k - k0) < (size_t)K1_CHUNK_K ? (k - k0) : (size_t)K1_CHUNK_K;
                p.k_begin = (int)k0;
                p.num_kb = (int)((kl + K1_BK - 1) / K1_BK);
                p.c = part + q * m * n;
                p.rsc = (int64_t)n;
                p.csc = 1;
                p.epi = LinearEpi{1, 0, MODE_NEAREST, OUT_I32};
                p.fast = (n % 4) == 0;
                e = k1_launch(tmA, tmB, false, true, p, grid, s);
            }
            if (e == cudaSuccess)
                e = reduce_chunks(part, (int)chunks, m, n, c, (int64_t)ldc, 1, epi, s);
        }
    }
    if (e != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    if (cudaStreamSynchronize(s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    int word = 0;
    if (cudaMemcpyAsync(&word, status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    return word ? UOR_B200_TIMEOUT : UOR_B200_OK;
}
