/*
 * fa_oracle.c -- fp64 CPU oracle for the SDPA forward.  TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
 * load this library.  The product path (fused_attn / libfa_sm100.so) never calls it, and there is
 * no CPU fallback built on it.
 *
 * What it restates (reference = yashpatil582/fused-attention-cuda):
 *   fa_oracle_rows       src/reference/cpu_reference.cpp:47-81   direct softmax of one head's rows
 *   fa_oracle_attention  src/reference/cpu_reference.cpp:83-92   whole tensor, (b, h) loop
 *   fa_oracle_tiled      src/reference/cpu_reference.cpp:94-165  tiled online-softmax recurrence
 *   fa_oracle_max_abs    src/reference/cpu_reference.cpp:167-175 NaN-aware max |a - b|
 * Conventions (src/reference/cpu_reference.h:9-14, include/fa/attention.cuh:28-40):
 *   q, o are [B, H, N, D]; k, v are [B, Hkv, N, D]; lse is [B, H, N]; all contiguous, D fastest.
 *   Query head h reads kv head h / (H / Hkv).  Causal is top-left aligned: key j is visible to
 *   query i iff j <= i.  A row with no visible key gets o = 0 and lse = +inf.
 *   lse = max_j(scale * s_ij) + ln(sum_j exp(scale * s_ij - max)), natural-log units.
 *
 * Differences from the reference that do not change any value: the (b, h, row-block) work items
 * are spread over POSIX threads (the reference harness does the same with std::thread over heads,
 * bench/bench_main.cu), and a second entry point with the tiled recurrence is exposed for the
 * tile-invariance tests.  The summation order inside one row is the reference's.
 *
 * Build: see oracle/Makefile (plain C11, no CUDA).
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct fa_oracle_shape {
  int B, H, Hkv, N, D;
  double scale;
  int causal;
} fa_oracle_shape;

static size_t head_base(const fa_oracle_shape* s, int heads, int b, int h, int n) {
  return (((size_t)b * (size_t)heads + (size_t)h) * (size_t)s->N + (size_t)n) * (size_t)s->D;
}

static int kv_head_of(const fa_oracle_shape* s, int h) { return h / (s->H / s->Hkv); }

static double dot(const double* a, const double* b, int d) {
  double acc = 0.0;
  for (int i = 0; i < d; ++i) acc += a[i] * b[i];
  return acc;
}

/* Rows [row0, row0 + rows) of head (b, h).  o: rows*D doubles, lse: rows doubles (or NULL).
 * `scores` is caller-provided scratch of N doubles.  cpu_reference.cpp:47-81. */
static void rows_impl(const double* q, const double* k, const double* v, const fa_oracle_shape* s,
                      int b, int h, int row0, int rows, double* o, double* lse, double* scores) {
  const int hk = kv_head_of(s, h);
  for (int r = 0; r < rows; ++r) {
    const int i = row0 + r;
    const double* qi = q + head_base(s, s->H, b, h, i);
    const int jmax = s->causal ? i : s->N - 1;
    double m = -INFINITY;
    for (int j = 0; j < s->N; ++j) {
      const double sc = (j <= jmax) ? s->scale * dot(qi, k + head_base(s, s->Hkv, b, hk, j), s->D)
                                    : -INFINITY;
      scores[j] = sc;
      if (sc > m) m = sc;
    }
    double* oi = o + (size_t)r * (size_t)s->D;
    memset(oi, 0, sizeof(double) * (size_t)s->D);
    if (m == -INFINITY) {
      if (lse) lse[r] = INFINITY;
      continue;
    }
    double l = 0.0;
    for (int j = 0; j <= jmax && j < s->N; ++j) {
      const double p = exp(scores[j] - m);
      l += p;
      const double* vj = v + head_base(s, s->Hkv, b, hk, j);
      for (int d = 0; d < s->D; ++d) oi[d] += p * vj[d];
    }
    for (int d = 0; d < s->D; ++d) oi[d] /= l;
    if (lse) lse[r] = m + log(l);
  }
}

void fa_oracle_rows(const double* q, const double* k, const double* v, const fa_oracle_shape* s,
                    int b, int h, int row0, int rows, double* o, double* lse) {
  double* scores = (double*)malloc(sizeof(double) * (size_t)s->N);
  if (!scores) return;
  rows_impl(q, k, v, s, b, h, row0, rows, o, lse, scores);
  free(scores);
}

/* ---- threaded whole-tensor driver ------------------------------------------------------ */

typedef struct work_ctx {
  const double *q, *k, *v;
  const fa_oracle_shape* s;
  double *o, *lse;
  int row_block;         /* rows per work item */
  int blocks_per_head;   /* ceil(N / row_block) */
  long long n_items;     /* B * H * blocks_per_head */
  long long next;        /* shared counter (atomic) */
} work_ctx;

static void* worker(void* arg) {
  work_ctx* c = (work_ctx*)arg;
  double* scores = (double*)malloc(sizeof(double) * (size_t)c->s->N);
  if (!scores) return NULL;
  for (;;) {
    const long long it = __atomic_fetch_add(&c->next, 1, __ATOMIC_RELAXED);
    if (it >= c->n_items) break;
    const int blk = (int)(it % c->blocks_per_head);
    const long long bh = it / c->blocks_per_head;
    const int b = (int)(bh / c->s->H), h = (int)(bh % c->s->H);
    const int row0 = blk * c->row_block;
    int rows = c->s->N - row0;
    if (rows > c->row_block) rows = c->row_block;
    double* ob = c->o + head_base(c->s, c->s->H, b, h, row0);
    double* lb = c->lse ? c->lse + (size_t)bh * (size_t)c->s->N + (size_t)row0 : NULL;
    rows_impl(c->q, c->k, c->v, c->s, b, h, row0, rows, ob, lb, scores);
  }
  free(scores);
  return NULL;
}

/* Whole tensor (cpu_reference.cpp:83-92) on `threads` POSIX threads (<= 1: calling thread).
 * Returns the number of threads actually used. */
int fa_oracle_attention(const double* q, const double* k, const double* v,
                        const fa_oracle_shape* s, double* o, double* lse, int threads) {
  work_ctx c;
  c.q = q, c.k = k, c.v = v, c.s = s, c.o = o, c.lse = lse;
  c.row_block = 64;
  c.blocks_per_head = (s->N + c.row_block - 1) / c.row_block;
  c.n_items = (long long)s->B * s->H * c.blocks_per_head;
  c.next = 0;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((long long)threads > c.n_items) threads = (int)(c.n_items > 0 ? c.n_items : 1);
  if (threads == 1) {
    worker(&c);
    return 1;
  }
  pthread_t tid[256];
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    if (pthread_create(&tid[t], NULL, worker, &c) == 0) ++started;
  }
  if (started == 0) worker(&c);
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
  return started == 0 ? 1 : started;
}

/* Tiled online-softmax recurrence (cpu_reference.cpp:94-165): block_m query rows x block_n keys,
 * running max m in RAW score units, c = scale*log2(e), alpha = 2^((m_old - m_new) c),
 * p = 2^((s - m_new) c), deferred 1/l, lse = m*scale + ln(l); causal key tiles that start past
 * the block's last query are skipped before any work.  `skip_masked` = 0 keeps those tiles
 * (every p is then 0), which the tests use to show the skip is exact. */
void fa_oracle_tiled(const double* q, const double* k, const double* v, const fa_oracle_shape* s,
                     int block_m, int block_n, int skip_masked, double* o, double* lse) {
  const double LOG2E = 1.4426950408889634;
  const double c = s->scale * LOG2E;
  double* m = (double*)malloc(sizeof(double) * (size_t)block_m);
  double* l = (double*)malloc(sizeof(double) * (size_t)block_m);
  double* acc = (double*)malloc(sizeof(double) * (size_t)block_m * (size_t)s->D);
  double* sc = (double*)malloc(sizeof(double) * (size_t)block_n);
  if (!m || !l || !acc || !sc) goto out;
  for (int b = 0; b < s->B; ++b) {
    for (int h = 0; h < s->H; ++h) {
      const int hk = kv_head_of(s, h);
      for (int bm = 0; bm < s->N; bm += block_m) {
        const int rows = (s->N - bm < block_m) ? s->N - bm : block_m;
        for (int r = 0; r < block_m; ++r) m[r] = -INFINITY, l[r] = 0.0;
        memset(acc, 0, sizeof(double) * (size_t)block_m * (size_t)s->D);
        for (int bn = 0; bn < s->N; bn += block_n) {
          if (skip_masked && s->causal && bn > bm + rows - 1) break;
          const int cols = (s->N - bn < block_n) ? s->N - bn : block_n;
          for (int r = 0; r < rows; ++r) {
            const int i = bm + r;
            const double* qi = q + head_base(s, s->H, b, h, i);
            double tmax = -INFINITY;
            for (int ci = 0; ci < cols; ++ci) {
              const int j = bn + ci;
              const double raw = (!s->causal || j <= i)
                                     ? dot(qi, k + head_base(s, s->Hkv, b, hk, j), s->D)
                                     : -INFINITY;
              sc[ci] = raw;
              if (raw > tmax) tmax = raw;
            }
            const double m_old = m[r];
            const double m_new = (tmax > m_old) ? tmax : m_old;
            if (m_new == -INFINITY) continue;
            const double alpha = (m_old == -INFINITY) ? 0.0 : exp2((m_old - m_new) * c);
            double* ar = acc + (size_t)r * (size_t)s->D;
            for (int d = 0; d < s->D; ++d) ar[d] *= alpha;
            double rowsum = 0.0;
            for (int ci = 0; ci < cols; ++ci) {
              const double p = (sc[ci] == -INFINITY) ? 0.0 : exp2((sc[ci] - m_new) * c);
              rowsum += p;
              const double* vj = v + head_base(s, s->Hkv, b, hk, bn + ci);
              for (int d = 0; d < s->D; ++d) ar[d] += p * vj[d];
            }
            l[r] = alpha * l[r] + rowsum;
            m[r] = m_new;
          }
        }
        for (int r = 0; r < rows; ++r) {
          const int i = bm + r;
          const double inv = (l[r] > 0.0) ? 1.0 / l[r] : 0.0;
          double* oi = o + head_base(s, s->H, b, h, i);
          const double* ar = acc + (size_t)r * (size_t)s->D;
          for (int d = 0; d < s->D; ++d) oi[d] = ar[d] * inv;
          if (lse) {
            lse[((size_t)b * s->H + h) * s->N + i] =
                (l[r] > 0.0 && m[r] != -INFINITY) ? m[r] * s->scale + log(l[r]) : INFINITY;
          }
        }
      }
    }
  }
out:
  free(m), free(l), free(acc), free(sc);
}

double fa_oracle_max_abs(const double* a, const double* b, size_t n) {
  double worst = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const double d = fabs(a[i] - b[i]);
    if (d != d) return INFINITY;
    if (d > worst) worst = d;
  }
  return worst;
}
