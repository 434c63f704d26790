/*
 * TEST INFRASTRUCTURE ONLY — the checker, never the product.
 *
 * CPU restatement of the arithmetic ml-edsl's CPU pipeline performs for
 * linalg.matmul and the dense layer relu(X @ W + b). Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm load
 * this library.
 *
 * Parity pinning: the reference itself cannot be built here (it needs
 * LLVM/MLIR >= 18, protoc and libomp, none present), so bit-level results are
 * unpinned; this restatement is pinned to every known answer the reference's
 * own tests hold for the path (tests/golden/), and to NumPy float64.
 *
 * What is restated, with the reference lines it follows:
 *  - C = 0 then C += A*B: linalg.fill(0) + linalg.matmul
 *      (cpp/src/builders/LinalgBuilder.cpp:118-138).
 *  - Schedule: 64x64 output tiles as parallel tasks (OpenMP in the reference,
 *      a pthread pool handing out tiles here), K untiled
 *      (cpp/src/MLIRLowering.cpp:366-375, MLIRLoweringPasses.cpp:470-473),
 *      8x8x8 inner tiles (MLIRLoweringPasses.cpp:467-469) with k ascending.
 *  - Static 8x8 tiles become vector.contract -> outer products -> vector.fma
 *      (MLIRLoweringPasses.cpp:103-185, MLIRLowering.cpp:385,401-407,422-424):
 *      one fused multiply-add per k, k ascending.
 *      Tiles whose shape is not static 8x8x8 fall back to scalar loops
 *      (MLIRLowering.cpp:410) computing a separate mulf then addf. Which case
 *      applies is decided per function (the tiled loop body is one region):
 *      static 8x8 tiles need M, N each a multiple of 64 (or a multiple of 8
 *      below 64) and K a multiple of 8. This rule is from reading the passes;
 *      it is not verified against a run of the reference.
 *  - Bias + activation in one pass after the full K sum, fused by
 *      linalg-fuse-elementwise-ops (MLIRLowering.cpp:355):
 *      y = act(acc + b[j]); relu = arith.maximumf(y, 0) (LinalgBuilder.cpp:213-215:
 *      NaN propagates, -0 -> +0); leaky = maximumf(y,0) + alpha*minimumf(y,0)
 *      (LinalgBuilder.cpp:216-225).
 *  - i32: arith.muli / arith.addi wrap modulo 2^32.
 * Build with -ffp-contract=off so that the MULADD path really rounds twice.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

enum { ACT_NONE = 0, ACT_RELU = 1, ACT_LEAKY = 2 };
enum { MODE_AUTO = -1, MODE_FMA = 0, MODE_MULADD = 1 };

static int dim_is_static8(int64_t d) { return (d % 64 == 0) || (d < 64 && d % 8 == 0); }

int oracle_fma_mode(int64_t M, int64_t N, int64_t K) {
  return (dim_is_static8(M) && dim_is_static8(N) && K % 8 == 0) ? MODE_FMA : MODE_MULADD;
}

static float maximumf0(float x) { return (x > 0.0f || isnan(x)) ? x : 0.0f; }
static float minimumf0(float x) { return (x < 0.0f || isnan(x)) ? x : 0.0f; }

static float act_apply(float y, int act, float alpha) {
  if (act == ACT_RELU) return maximumf0(y);
  if (act == ACT_LEAKY) {
    float pos = maximumf0(y);
    float neg = minimumf0(y) * alpha;
    return pos + neg;
  }
  return y;
}

/* Parallel-for over [0, n) tasks on `nthreads` threads (0 = all online
 * cores); tasks are handed out one at a time from an atomic counter. */
typedef void (*task_fn)(void* ctx, int64_t task);
typedef struct {
  task_fn fn;
  void* ctx;
  int64_t n;
  atomic_llong next;
} pool_t;

static void* pool_worker(void* arg) {
  pool_t* p = (pool_t*)arg;
  for (;;) {
    int64_t t = atomic_fetch_add(&p->next, 1);
    if (t >= p->n) break;
    p->fn(p->ctx, t);
  }
  return NULL;
}

static void parallel_for(int64_t n, int nthreads, task_fn fn, void* ctx) {
  if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > n) nthreads = (int)(n > 0 ? n : 1);
  pool_t p;
  p.fn = fn;
  p.ctx = ctx;
  p.n = n;
  atomic_init(&p.next, 0);
  pthread_t th[256];
  for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, pool_worker, &p);
  pool_worker(&p);
  for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
}

int oracle_default_threads(void) { return (int)sysconf(_SC_NPROCESSORS_ONLN); }

typedef struct {
  const float *X, *W, *b;
  float* Y;
  int64_t M, N, K, tn;
  int act, mode;
  float alpha;
} dense_ctx;

static void dense_tile(void* vctx, int64_t task) {
  const dense_ctx* c = (const dense_ctx*)vctx;
  const int64_t M = c->M, N = c->N, K = c->K;
  const int64_t i0 = (task / c->tn) * 64, j0 = (task % c->tn) * 64;
  const int64_t ni = (M - i0 < 64) ? M - i0 : 64;
  const int64_t nj = (N - j0 < 64) ? N - j0 : 64;
  float acc[64][64];
  memset(acc, 0, sizeof acc); /* linalg.fill(0) */
  for (int64_t k = 0; k < K; ++k) {
    const float* brow = c->W + k * N + j0;
    for (int64_t i = 0; i < ni; ++i) {
      const float a = c->X[(i0 + i) * K + k];
      float* cr = acc[i];
      if (c->mode == MODE_FMA) {
        for (int64_t j = 0; j < nj; ++j) cr[j] = fmaf(a, brow[j], cr[j]);
      } else {
        for (int64_t j = 0; j < nj; ++j) {
          const float p = a * brow[j];
          cr[j] = cr[j] + p;
        }
      }
    }
  }
  for (int64_t i = 0; i < ni; ++i)
    for (int64_t j = 0; j < nj; ++j) {
      float y = acc[i][j];
      if (c->b) y = y + c->b[j0 + j];
      c->Y[(i0 + i) * N + j0 + j] = act_apply(y, c->act, c->alpha);
    }
}

/* Y[M,N] = act(X[M,K] @ W[K,N] (+ b)). Row-major, contiguous. */
void oracle_dense_f32(const float* X, const float* W, const float* b, float* Y, int64_t M,
                      int64_t N, int64_t K, int act, float alpha, int mode, int nthreads) {
  if (mode == MODE_AUTO) mode = oracle_fma_mode(M, N, K);
  dense_ctx c = {X, W, b, Y, M, N, K, (N + 63) / 64, act, mode, alpha};
  parallel_for(((M + 63) / 64) * c.tn, nthreads, dense_tile, &c);
}

typedef struct {
  const int32_t *A, *B, *bias;
  int32_t* C;
  int64_t M, N, K;
} i32_ctx;

static void i32_row(void* vctx, int64_t i) {
  const i32_ctx* c = (const i32_ctx*)vctx;
  const int64_t N = c->N, K = c->K;
  uint32_t* crow = (uint32_t*)(c->C + i * N);
  for (int64_t j = 0; j < N; ++j) crow[j] = 0u;
  for (int64_t k = 0; k < K; ++k) {
    const uint32_t a = (uint32_t)c->A[i * K + k];
    const int32_t* brow = c->B + k * N;
    for (int64_t j = 0; j < N; ++j) crow[j] += a * (uint32_t)brow[j];
  }
  if (c->bias)
    for (int64_t j = 0; j < N; ++j) crow[j] += (uint32_t)c->bias[j];
}

/* C[M,N] = A[M,K] @ B[K,N] (+ bias) modulo 2^32. */
void oracle_matmul_i32(const int32_t* A, const int32_t* B, const int32_t* bias, int32_t* C,
                       int64_t M, int64_t N, int64_t K, int nthreads) {
  i32_ctx c = {A, B, bias, C, M, N, K};
  parallel_for(M, nthreads, i32_row, &c);
}

/* Y = act(X + b) (b may be NULL), the standalone bias_add / relu generics. */
void oracle_bias_act_f32(const float* X, const float* b, float* Y, int64_t M, int64_t N, int act,
                         float alpha) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      float y = X[i * N + j];
      if (b) y = y + b[j];
      Y[i * N + j] = act_apply(y, act, alpha);
    }
}

/* ---- 1-D reductions and dot: the sequential fold linalg.reduce / linalg.dot
 * define. dot: 0-D accumulator filled with 0, acc = acc + a[i]*b[i] with the
 * product rounded first (cpp/src/builders/LinalgBuilder.cpp:66-104).
 * reduce: acc = init, then acc = body(x[i], acc) for i ascending
 * (LinalgBuilder.cpp:241-279) with the library's bodies
 * (mlir_edsl/ops/linalg.py:104-175): sum acc + x, product acc * x,
 * max If(x > acc, x, acc), min If(x < acc, x, acc). */
enum { RED_SUM = 0, RED_PROD = 1, RED_MAX = 2, RED_MIN = 3 };

float oracle_reduce_f32(const float* x, int64_t n, int op, float init) {
  float acc = init;
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    if (op == RED_SUM) acc = acc + v;
    else if (op == RED_PROD) acc = acc * v;
    else if (op == RED_MAX) acc = (v > acc) ? v : acc;
    else acc = (v < acc) ? v : acc;
  }
  return acc;
}

int32_t oracle_reduce_i32(const int32_t* x, int64_t n, int op, int32_t init) {
  uint32_t acc = (uint32_t)init;
  for (int64_t i = 0; i < n; ++i) {
    const int32_t v = x[i];
    if (op == RED_SUM) acc += (uint32_t)v;
    else if (op == RED_PROD) acc *= (uint32_t)v;
    else if (op == RED_MAX) acc = (v > (int32_t)acc) ? (uint32_t)v : acc;
    else acc = (v < (int32_t)acc) ? (uint32_t)v : acc;
  }
  return (int32_t)acc;
}

float oracle_dot_f32(const float* a, const float* b, int64_t n) {
  float acc = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    const float p = a[i] * b[i];
    acc = acc + p;
  }
  return acc;
}

int32_t oracle_dot_i32(const int32_t* a, const int32_t* b, int64_t n) {
  uint32_t acc = 0u;
  for (int64_t i = 0; i < n; ++i) acc += (uint32_t)a[i] * (uint32_t)b[i];
  return (int32_t)acc;
}
