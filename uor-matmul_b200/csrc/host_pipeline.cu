// host_pipeline.cu -- host-pointer calls of the exact i8 GEMM with the PCIe copies
// overlapped with each other and with the tensor-core work.
//
// The output is tiled into blocks; A row blocks and B column blocks go up on one copy
// stream in the order the blocks need them, each block is computed on the context's
// stream as soon as its operands have landed, and each finished C block comes back on
// a second copy stream while later blocks are still arriving and computing. Every
// block is the same exact GEMM over the full reduction, so the bytes are those of the
// unpipelined call.
#include "int_gemm.h"
#include <algorithm>
#include "staging.h"

namespace uor {

static cudaEvent_t ctx_event(uor_b200_ctx* ctx, int i, int* st) {
    while (ctx->nevents <= i) {
        if (ctx->nevents >= 256 ||
            cudaEventCreateWithFlags(&ctx->events[ctx->nevents], cudaEventDisableTiming) !=
                cudaSuccess) {
            *st = UOR_B200_DEVICE_ERROR;
            return nullptr;
        }
        ++ctx->nevents;
    }
    return ctx->events[i];
}

bool i8_pipeline_applies(const Operand& A, const Operand& B, const Operand& C) {
    const size_t m = A.rows, k = A.cols, n = B.cols;
    if (m * n < (size_t)4 << 20 || k == 0) return false;
    // Row-major operands whose blocks stay 16-byte aligned on the device, so every
    // block runs the TMA path without a gather.
    return k % 16 == 0 && n % 16 == 0 && A.cs == 1 && A.rs >= (ptrdiff_t)k && B.cs == 1 &&
           B.rs >= (ptrdiff_t)n && C.cs == 1 && C.rs >= (ptrdiff_t)n;
}

int run_i8_gemm_pipelined(uor_b200_ctx* ctx, const Operand& A, const Operand& B, const Operand& C,
                          const LinearEpi& epi, uor_b200_route* route) {
    const size_t m = A.rows, k = A.cols, n = B.cols, ob = C.es;
    int st = UOR_B200_OK;
    if (!ctx->copy_in &&
        (cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking) != cudaSuccess ||
         cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking) != cudaSuccess))
        return UOR_B200_DEVICE_ERROR;
    auto* da = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_A, m * k, &st));
    if (!da) return st;
    auto* db = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_B, k * n, &st));
    if (!db) return st;
    auto* dc = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_C, m * n * ob, &st));
    if (!dc) return st;
    // About 2048 x 2048 blocks, at most 8 x 8 of them; block edges on 256-cell tiles.
    // Smaller blocks start the copy-out earlier but cost more in short copy rows and
    // launches than they win (8192^3 from pinned memory: 5.85 ms at 2048, 6.46 ms at
    // 1024, 7.48 ms unpipelined). Only the first row of blocks is cut finer: its first
    // column block is split into quarter, quarter and half widths, so that the first
    // copy-out waits for one A row block and a quarter of a B column block instead of a
    // whole one. With row blocks of k/4 rows or more, each further B piece brings as
    // many bytes of output as of input, so the copy-out stream stays busy from then on.
    auto blocks = [](size_t x) { return (int)std::min<size_t>(8, (x + 2047) / 2048); };
    const int R = blocks(m), S = blocks(n);
    const size_t rb = (m + R - 1) / R + 255 & ~(size_t)255;
    const size_t cb = (n + S - 1) / S + 255 & ~(size_t)255;
    // B pieces in copy order: column ranges [pc[i], pc[i + 1]).
    size_t pc[12];
    int P = 0;
    pc[0] = 0;
    const size_t q = cb / 4 & ~(size_t)255;
    if (S > 1 && q >= 256) {
        pc[++P] = q;
        pc[++P] = 2 * q;
    }
    for (size_t c0 = cb; c0 < n; c0 += cb) pc[++P] = c0;
    pc[++P] = n;
    const auto* ha = A.origin;
    const auto* hb = B.origin;
    auto* hc = const_cast<uint8_t*>(C.origin);
    cudaStream_t in = ctx->copy_in, out = ctx->copy_out, cs = ctx->stream;
    // events: [0, R) A row blocks, [R, R + P) B pieces, then per C block: C-in, C-done
    auto ev = [&](int i) { return ctx_event(ctx, i, &st); };
    const int nblk = P + (R - 1) * S;
    for (int i = 0; i < R + P + 2 * nblk; ++i)
        if (!ev(i)) return st;
    const bool reads_c = epi.beta != 0;
    cudaPointerAttributes pa{};
    const bool pinned_out =
        cudaPointerGetAttributes(&pa, hc) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();  // an unregistered pointer is not an error here
    // The input stream must not overtake work already queued on the compute stream
    // that reads these buffers (a previous call).
    if (cudaEventRecord(ev(0), cs) != cudaSuccess || cudaStreamWaitEvent(in, ev(0), 0) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    auto put_a = [&](int r) {
        const size_t r0 = std::min(r * rb, m), mr = std::min(rb, m - r0);
        if (mr)
            cudaMemcpy2DAsync(da + r0 * k, k, ha + r0 * A.rs, A.rs, k, mr, cudaMemcpyHostToDevice,
                              in);
        cudaEventRecord(ev(r), in);
    };
    auto put_b = [&](int i) {
        const size_t c0 = pc[i], nc = pc[i + 1] - pc[i];
        if (nc) cudaMemcpy2DAsync(db + c0, n, hb + c0, B.rs, nc, k, cudaMemcpyHostToDevice, in);
        cudaEventRecord(ev(R + i), in);
    };
    put_a(0);
    for (int i = 0; i < P; ++i) put_b(i);
    for (int r = 1; r < R; ++r) put_a(r);
    // Copies already queued must finish before the host buffers are handed back, also
    // when a block fails to launch.
    auto drain = [&](int status) {
        cudaStreamSynchronize(in);
        cudaStreamSynchronize(cs);
        cudaStreamSynchronize(out);
        return status;
    };
    // The C blocks in launch order: the pieces along the first row, whole blocks after.
    struct Blk {
        size_t r0, mr, c0, nc;
        int a_ev, b_ev;
    };
    auto block_at = [&](int i) {
        Blk b{};
        if (i < P) {
            b = {0, std::min(rb, m), pc[i], pc[i + 1] - pc[i], 0, R + i};
        } else {
            const int r = 1 + (i - P) / S, c = (i - P) % S;
            b.r0 = std::min(r * rb, m);
            b.mr = std::min(rb, m - b.r0);
            b.c0 = std::min(c * cb, n);
            b.nc = std::min(cb, n - b.c0);
            b.a_ev = r;  // queued after every B piece
            b.b_ev = -1;
        }
        return b;
    };
    for (int i = 0; i < nblk; ++i) {
        const Blk bk = block_at(i);
        if (!bk.mr || !bk.nc) continue;
        uint8_t* dcb = dc + (bk.r0 * n + bk.c0) * ob;
        uint8_t* hcb = hc + (bk.r0 * C.rs + bk.c0) * ob;
        if (reads_c) {
            cudaMemcpy2DAsync(dcb, n * ob, hcb, C.rs * ob, bk.nc * ob, bk.mr,
                              cudaMemcpyHostToDevice, in);
            cudaEventRecord(ev(R + P + 2 * i), in);
            cudaStreamWaitEvent(cs, ev(R + P + 2 * i), 0);
        }
        cudaStreamWaitEvent(cs, ev(bk.a_ev), 0);
        if (bk.b_ev >= 0) cudaStreamWaitEvent(cs, ev(bk.b_ev), 0);
        uor_b200_route sub{};
        st = run_i8_gemm(ctx, reinterpret_cast<const int8_t*>(da + bk.r0 * k), (ptrdiff_t)k, 1,
                         reinterpret_cast<const int8_t*>(db + bk.c0), (ptrdiff_t)n, 1, dcb,
                         (ptrdiff_t)n, 1, bk.mr, k, bk.nc, epi, &sub);
        if (st) return drain(st);
        if (route && i == 0) *route = sub;
        cudaEventRecord(ev(R + P + 2 * i + 1), cs);
        if (pinned_out) {
            cudaStreamWaitEvent(out, ev(R + P + 2 * i + 1), 0);
            cudaMemcpy2DAsync(hcb, C.rs * ob, dcb, n * ob, bk.nc * ob, bk.mr,
                              cudaMemcpyDeviceToHost, out);
        }
    }
    // Into pageable memory a copy-out returns only when it is done: queue those after
    // every block, so that they do not hold back the launches behind them.
    for (int i = 0; i < nblk && !pinned_out; ++i) {
        const Blk bk = block_at(i);
        if (!bk.mr || !bk.nc) continue;
        cudaStreamWaitEvent(out, ev(R + P + 2 * i + 1), 0);
        cudaMemcpy2DAsync(hc + (bk.r0 * C.rs + bk.c0) * ob, C.rs * ob, dc + (bk.r0 * n + bk.c0) * ob,
                          n * ob, bk.nc * ob, bk.mr, cudaMemcpyDeviceToHost, out);
    }
    if (cudaGetLastError() != cudaSuccess) return drain(UOR_B200_DEVICE_ERROR);
    if (cudaStreamSynchronize(out) != cudaSuccess) return drain(UOR_B200_DEVICE_ERROR);
    return uor_b200_ctx_sync(ctx);
}

}  // namespace uor
