// capi_arena.cu -- the Arena tier's C ABI (crates/uor-matmul-codec/src/codecs.rs:894-1028):
// codes of one byte or two index a table of N float symbols (bit patterns) modulo N, and
// the product of a float A with the decoded matrix is the exact float GEMM of the float
// family (run_float_gemm). canonicalize's host helper builds such a table.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>
#include "float_exact.h"
#include "internal.h"
#include "staging.h"
#include "walk.cuh"

using namespace uor;

namespace {

// Arena::decode_element (codecs.rs:961-965): table[code % N], one element per code, at
// CodedMatrix::at's position (matrix.rs:202-207) with a one-element block. The symbols
// move as bit patterns (W = uint32_t for f32, uint64_t for f64); the output is the dense
// k x n row-major B the float path reads.
template <typename W>
__global__ void arena_decode_kernel(W* __restrict__ out, const uint8_t* __restrict__ codes,
                                    const W* __restrict__ table, uint32_t N, int cb,
                                    int orientation, int k, int n) {
    const int64_t total = static_cast<int64_t>(k) * n;
    for (GridWalk wk(static_cast<size_t>(n)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int64_t idx = static_cast<int64_t>(wk.idx);
        const int p = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        const int64_t at = orientation == 0 ? idx : static_cast<int64_t>(j) * k + p;
        const uint32_t code =
            cb == 1 ? codes[at]
                    : (static_cast<uint32_t>(codes[2 * at]) | static_cast<uint32_t>(codes[2 * at + 1]) << 8);
        out[idx] = table[code % N];
    }
}

// The same decode for codes laid n x k (gemm_tabulated's W), through a 32 x 32 shared tile:
// codes are read along k and symbols written along n, both coalesced.
template <typename W>
__global__ void arena_decode_t_kernel(W* __restrict__ out, const uint8_t* __restrict__ codes,
                                      const W* __restrict__ table, uint32_t N, int cb, int k, int n) {
    __shared__ uint32_t tile[32][33];
    const int p0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int r = ty; r < 32; r += 8) {
        const int j = j0 + r, p = p0 + tx;
        uint32_t code = 0;
        if (j < n && p < k) {
            const int64_t at = static_cast<int64_t>(j) * k + p;
            code = cb == 1 ? codes[at]
                           : (static_cast<uint32_t>(codes[2 * at]) | static_cast<uint32_t>(codes[2 * at + 1]) << 8);
        }
        tile[r][tx] = code;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int p = p0 + r, j = j0 + tx;
        if (p < k && j < n) out[static_cast<int64_t>(p) * n + j] = table[tile[tx][r] % N];
    }
}

bool float_type(uor_b200_dtype t) { return t == UOR_B200_F32 || t == UOR_B200_F64; }

int arena_common(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                 const void* table, size_t table_len, const uint8_t* codes, size_t codes_len,
                 uint32_t code_bytes, size_t k, size_t n, uint32_t orientation,
                 const uor_b200_view_mut* c, int64_t alpha, int64_t beta,
                 const uor_b200_call* call) {
    if (!a || !c || orientation > 1) return UOR_B200_INVALID_ARGUMENT;
    if (!float_type(elem) || !float_type(out)) return UOR_B200_UNSUPPORTED;
    if (code_bytes != 1 && code_bytes != 2) return UOR_B200_INVALID_ARGUMENT;
    if (!table || table_len == 0) return UOR_B200_INVALID_ARGUMENT;
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    // CodedMatrix::new (matrix.rs:36-60): exactly one code per element of the shape.
    const size_t rows = orientation == 0 ? k : n, cols = orientation == 0 ? n : k;
    if (rows * cols * code_bytes != codes_len) return UOR_B200_DOES_NOT_FIT;
    const size_t es = dtype_size(elem);
    Operand A, C;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, es, &A))) return st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)))
        return st;
    if (a->cols != k || c->rows != a->rows || c->cols != n) return UOR_B200_NONCONFORMANT;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    uor_b200_route local{};
    uor_b200_route* route = call && call->route ? call->route : &local;
    *route = uor_b200_route{};
    const size_t m = a->rows;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    if (codes_len && !codes) return UOR_B200_INVALID_ARGUMENT;
    const bool dev = call && (call->flags & UOR_B200_DEVICE_POINTERS);

    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    cudaStream_t s = ctx->stream;
    const uint8_t* da = nullptr;
    OutStage cs;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da))) return st;
    const uint8_t* dcodes = codes;
    if (!dev && codes_len) {
        uint8_t* d = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_B, codes_len, &st));
        if (!d) return st;
        if (cudaMemcpyAsync(d, codes, codes_len, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        dcodes = d;
    }
    if ((st = stage_out_begin(ctx, C, dev, beta != 0, &cs))) return st;
    // The table, then the dense decoded B, in the decoded-operand slot (the float
    // driver uses the workspace and auxiliary slots itself).
    const size_t tbytes = (table_len * es + 255) / 256 * 256;
    uint8_t* buf = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_DECODED, tbytes + k * n * es + 256, &st));
    if (!buf) return st;
    if (cudaMemcpyAsync(buf, table, table_len * es,
                        dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    uint8_t* dense = buf + tbytes;
    if (k) {
        const int64_t total = (int64_t)k * n;
        const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
        const uint32_t N = table_len > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)table_len;
        const dim3 tg((unsigned)((k + 31) / 32), (unsigned)((n + 31) / 32));
        if (orientation == 1 && n <= 65535 * 32) {
            if (es == 4)
                arena_decode_t_kernel<uint32_t><<<tg, dim3(32, 8), 0, s>>>(
                    reinterpret_cast<uint32_t*>(dense), dcodes, reinterpret_cast<const uint32_t*>(buf), N,
                    (int)code_bytes, (int)k, (int)n);
            else
                arena_decode_t_kernel<uint64_t><<<tg, dim3(32, 8), 0, s>>>(
                    reinterpret_cast<uint64_t*>(dense), dcodes, reinterpret_cast<const uint64_t*>(buf), N,
                    (int)code_bytes, (int)k, (int)n);
        } else if (es == 4)
            arena_decode_kernel<uint32_t><<<grid, 256, 0, s>>>(
                reinterpret_cast<uint32_t*>(dense), dcodes, reinterpret_cast<const uint32_t*>(buf), N,
                (int)code_bytes, (int)orientation, (int)k, (int)n);
        else
            arena_decode_kernel<uint64_t><<<grid, 256, 0, s>>>(
                reinterpret_cast<uint64_t*>(dense), dcodes, reinterpret_cast<const uint64_t*>(buf), N,
                (int)code_bytes, (int)orientation, (int)k, (int)n);
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    }
    st = run_float_gemm(ctx, elem == UOR_B200_F64, out == UOR_B200_F64, da, A.rs, A.cs, dense,
                        (ptrdiff_t)n, 1, cs.dev_origin, C.rs, C.cs, m, k, n, alpha, beta, mode,
                        route);
    if (st) return st;
    route->b_layout = 3;  // decoded to a dense workspace first
    if (!dev && (st = uor_b200_ctx_sync(ctx))) return st;  // the host table was read
    if ((st = stage_out_end(ctx, cs))) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

// canonicalize (codecs.rs:990-1003): unsigned order on bit patterns, distinct patterns
// moved to the front in that order; positions past the count keep the sorted stream's
// values there, as the reference's in-place compaction leaves them.
template <typename W>
size_t canonicalize_bits(W* v, size_t len) {
    std::sort(v, v + len);
    size_t n = 0;
    for (size_t i = 0; i < len; ++i)
        if (n == 0 || v[i] != v[n - 1]) v[n++] = v[i];
    return n;
}

}  // namespace

extern "C" {

int uor_b200_arena_gemm(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                        const void* table, size_t table_len, const uint8_t* codes,
                        size_t codes_len, uint32_t code_bytes, size_t k, size_t n,
                        uint32_t orientation, const uor_b200_view_mut* c, int64_t alpha,
                        int64_t beta, const uor_b200_call* call) {
    return arena_common(elem, out, a, table, table_len, codes, codes_len, code_bytes, k, n,
                        orientation, c, alpha, beta, call);
}

int uor_b200_arena_canonicalize(uor_b200_dtype elem, void* values, size_t len, size_t* distinct) {
    if (!distinct || (len && !values)) return UOR_B200_INVALID_ARGUMENT;
    if (elem == UOR_B200_F32)
        *distinct = canonicalize_bits(static_cast<uint32_t*>(values), len);
    else if (elem == UOR_B200_F64)
        *distinct = canonicalize_bits(static_cast<uint64_t*>(values), len);
    else
        return UOR_B200_UNSUPPORTED;
    return UOR_B200_OK;
}

}  // extern "C"
