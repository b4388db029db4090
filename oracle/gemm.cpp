// oracle/gemm.cpp -- multithreaded FP32 GEMM core for the CPU oracle.
//
// TEST INFRASTRUCTURE ONLY: this file is part of the parity oracle and the
// timed CPU baseline. The product path (rokoko_b200/) never links or calls it.
//
// C[M,N] (+)= A[M,K] * B[K,N], all row-major FP32 with explicit leading
// dimensions.  A 6x16 register-blocked micro-kernel written with GCC vector
// extensions; built with -mavx2 -mfma -ffp-contract=fast so the inner update is
// one FMA per element.  Rows of A may be given through an indirection table so
// that convolution taps (shifted, zero-padded rows) need no im2col copy.
#include "oracle_internal.h"

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace orc {

// ---------------------------------------------------------------- thread pool
namespace {
struct Pool {
    std::vector<std::thread> workers;
    std::mutex mu;
    std::condition_variable cv, done_cv;
    std::function<void(int)> job;
    int njobs = 0;
    std::atomic<int> next{0};
    int pending = 0;
    uint64_t gen = 0;
    bool stop = false;

    explicit Pool(int n) {
        for (int i = 0; i < n; i++) workers.emplace_back([this] { loop(); });
    }
    ~Pool() {
        { std::lock_guard<std::mutex> g(mu); stop = true; }
        cv.notify_all();
        for (auto& t : workers) t.join();
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return stop || gen != seen; });
            if (stop) return;
            seen = gen;
            lk.unlock();
            drain();
            lk.lock();
            if (--pending == 0) done_cv.notify_all();
        }
    }
    void drain() {
        for (;;) {
            int i = next.fetch_add(1);
            if (i >= njobs) break;
            job(i);
        }
    }
    void run(int n, const std::function<void(int)>& f) {
        if (n <= 0) return;
        if (workers.empty() || n == 1) { for (int i = 0; i < n; i++) f(i); return; }
        {
            std::lock_guard<std::mutex> g(mu);
            job = f; njobs = n; next = 0; pending = (int)workers.size(); gen++;
        }
        cv.notify_all();
        drain();
        std::unique_lock<std::mutex> lk(mu);
        done_cv.wait(lk, [&] { return pending == 0; });
    }
};

std::mutex g_pool_mu;
Pool* g_pool = nullptr;
int g_threads = 1;
}  // namespace

void set_threads(int n) {
    std::lock_guard<std::mutex> g(g_pool_mu);
    if (n < 1) n = 1;
    if (g_pool && g_threads == n) return;
    delete g_pool;
    g_pool = n > 1 ? new Pool(n - 1) : nullptr;
    g_threads = n;
}

int get_threads() { return g_threads; }

void parallel_for(int n, const std::function<void(int)>& f) {
    if (g_pool && n > 1) g_pool->run(n, f);
    else for (int i = 0; i < n; i++) f(i);
}

// ---------------------------------------------------------------- micro-kernel
typedef float v8 __attribute__((vector_size(32)));

static inline v8 ld8(const float* p) { v8 r; std::memcpy(&r, p, 32); return r; }
static inline void st8(float* p, v8 v) { std::memcpy(p, &v, 32); }
static inline v8 bc8(float x) { return (v8){x, x, x, x, x, x, x, x}; }

// C rows [r0, r0+mr) x cols [c0, c0+16) += sum_k A[row][k] * B[k][c]
// arow[i] points at A row (nullptr = zero row).
static void kern_6x16(int mr, int K, const float* const* arow, const float* B, int ldb,
                      float* const* crow, int c0) {
    v8 acc[6][2];
    for (int i = 0; i < 6; i++) { acc[i][0] = bc8(0.f); acc[i][1] = bc8(0.f); }
    const float* a[6];
    static const float zero_row[1] = {0.f};
    bool live[6];
    for (int i = 0; i < 6; i++) {
        live[i] = i < mr && arow[i] != nullptr;
        a[i] = live[i] ? arow[i] : zero_row;
    }
    for (int k = 0; k < K; k++) {
        const float* b = B + (size_t)k * ldb + c0;
        v8 b0 = ld8(b), b1 = ld8(b + 8);
#define ROW(i) if (live[i]) { v8 av = bc8(a[i][k]); acc[i][0] += av * b0; acc[i][1] += av * b1; }
        ROW(0) ROW(1) ROW(2) ROW(3) ROW(4) ROW(5)
#undef ROW
    }
    for (int i = 0; i < mr; i++) {
        float* c = crow[i] + c0;
        st8(c, ld8(c) + acc[i][0]);
        st8(c + 8, ld8(c + 8) + acc[i][1]);
    }
}

static void kern_scalar(int mr, int K, const float* const* arow, const float* B, int ldb,
                        float* const* crow, int c0, int c1) {
    for (int i = 0; i < mr; i++) {
        if (!arow[i]) continue;
        for (int c = c0; c < c1; c++) {
            float s = 0.f;
            for (int k = 0; k < K; k++) s += arow[i][k] * B[(size_t)k * ldb + c];
            crow[i][c] += s;
        }
    }
}

// C[m][:] += A_row(m) . B   for m in [0, M); A rows via `arow`, C rows via `crow`.
void gemm_rows_acc(int M, int N, int K, const float* const* arow, const float* B, int ldb,
                   float* const* crow) {
    const int MB = 6;
    const int KC = 256;  // K blocking keeps the B panel in L2
    int nblk = (M + MB - 1) / MB;
    int n16 = N / 16 * 16;
    // split columns too when rows are few
    int ncol_chunks = 1;
    if (nblk < 4 * get_threads() && n16 >= 64) ncol_chunks = std::min(n16 / 16, 8);
    int col_per = (n16 / 16 + ncol_chunks - 1) / ncol_chunks * 16;
    int rows_per_task = std::max(1, std::min(8, nblk / std::max(1, 2 * get_threads())));
    int ntask_r = (nblk + rows_per_task - 1) / rows_per_task;
    parallel_for(ntask_r * ncol_chunks, [&](int task) {
        int tr = task / ncol_chunks, tc = task % ncol_chunks;
        int cb0 = tc * col_per, cb1 = std::min(n16, cb0 + col_per);
        for (int rb = tr * rows_per_task; rb < std::min(nblk, (tr + 1) * rows_per_task); rb++) {
            int m0 = rb * MB, mr = std::min(MB, M - m0);
            for (int k0 = 0; k0 < K; k0 += KC) {
                int kc = std::min(KC, K - k0);
                const float* ap[MB];
                for (int i = 0; i < mr; i++) ap[i] = arow[m0 + i] ? arow[m0 + i] + k0 : nullptr;
                for (int i = mr; i < MB; i++) ap[i] = nullptr;
                const float* Bk = B + (size_t)k0 * ldb;
                for (int c = cb0; c < cb1; c += 16) kern_6x16(mr, kc, ap, Bk, ldb, crow + m0, c);
                if (tc == ncol_chunks - 1 && n16 < N) kern_scalar(mr, kc, ap, Bk, ldb, crow + m0, n16, N);
            }
        }
    });
}

void gemm_acc(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C, int ldc) {
    std::vector<const float*> ar(M);
    std::vector<float*> cr(M);
    for (int m = 0; m < M; m++) { ar[m] = A + (size_t)m * lda; cr[m] = C + (size_t)m * ldc; }
    gemm_rows_acc(M, N, K, ar.data(), B, ldb, cr.data());
}

}  // namespace orc
