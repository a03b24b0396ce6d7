/*
 * CPU oracle of the block-Gibbs group step — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's group kernel math, used by the
 * tests, the smoke check and the CPU baseline of bench.py as the checker; it
 * is never part of the product path.
 *
 * State is float32 [rows][n_chains] (the reference's flat float32 global
 * state of tt_thrml/executor.py:104-127 with a chain axis).  One call
 * performs one sampling group:
 *   - every block of the group is sampled from the same input state and all
 *     are committed afterwards (tt_thrml/compiler.py:436-450);
 *   - a block's field sums, interaction by interaction in program order, the
 *     terms of that interaction in order, each term = selected weight x
 *     product of the non-categorical sources (tt_thrml/compiler.py:274-318);
 *     categorical sources select the weight slice of their value
 *     (tt_thrml/compiler.py:289-300);
 *   - spin: +1 where 2*gamma > l (compiler.py:321-324); categorical:
 *     argmax(theta + g), first maximum (compiler.py:327-344), or in Philox
 *     mode the inverse-CDF draw of softmax(theta) from one uniform; gaussian:
 *     mean + sqrt(var)*xi with var = 1/(precision + 1e-6) (compiler.py:347-365).
 *
 * Variates: either given per block (the reference's uploaded slices,
 * tt_thrml/rng.py:132-222) or drawn from Philox4x32-10 (Salmon et al., SC'11)
 * with the same counter layout as the CUDA kernels; in Philox mode the spin
 * and categorical decisions are taken exactly in double precision and the
 * distance to the decision boundary is reported in `margin` so a checker can
 * tell a real mismatch from a threshold tie.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_SPIN 0
#define OR_CATEGORICAL 1
#define OR_GAUSSIAN 2
#define OR_KIND_PRECISION 1
#define OR_MAXQ 64

typedef struct {
  const int64_t* row_ptr;
  const float* weights;   /* [nnz][w_inner] */
  const int32_t* sources; /* [n_sources][nnz] */
  int64_t nnz;
  int32_t n_sources, n_categorical, kind, w_inner;
  int32_t cat_q[4];
} or_interaction;

/* rng_layout 0: counter (chain/4, row, sweep), word chain % 4, as the sparse,
 * generic and Potts kernels draw; 1: counter (chain, row/4, sweep), word
 * row % 4, as the dense tensor-core kernel draws (four consecutive rows of one
 * chain per counter).  Layouts 2 and 3 are the lattice kernels' split
 * uniforms (spin blocks): the 23-bit draw m = (h << 7) | f with h = 16 bits
 * of a shared counter "LSPI" and f = word 0 >> 25 of the draw's own counter
 * (chain, row, sweep, "LREF"); 2: counter (chain, row/8, sweep), half row % 2
 * of word (row/2) % 4 (the single-chain lattice stencil kernel); 3: counter
 * (chain/8, row, sweep), half chain % 2 of word (chain/2) % 4 (the
 * shared-memory resident lattice kernel).  Layout 4 ("planes", the bit-sliced
 * lattice kernel): bit 22 - b of m is bit 8 (row % 4) + (row % 32) / 4 of word
 * b % 4 of counter (chain, row / 32, sweep, "LPL0" + b / 4).  Layout 5
 * ("planes8", the bit-sliced resident kernel): bit 22 - b of m is bit
 * 8 (row % 4) + chain % 8 of word b % 4 of counter (chain / 8, row / 4,
 * sweep, "LPL0" + b / 4). */
typedef struct {
  int32_t family, q, n_interactions, rng_layout;
  int64_t n_nodes, row_start;
  const or_interaction* inter;
  const float* variates; /* this sweep: [n_nodes][qv][C], or NULL */
} or_block;

/* ---- Philox4x32-10 ---- */
typedef struct {
  uint32_t v[4];
} or_u32x4;

static or_u32x4 or_philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {
  or_u32x4 c = {{c0, c1, c2, c3}};
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.v[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.v[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    or_u32x4 n = {{hi1 ^ c.v[1] ^ k0, lo1, hi0 ^ c.v[3] ^ k1, lo0}};
    c = n;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  or_u32x4 r = or_philox(ctr[0], ctr[1], ctr[2], ctr[3], key[0], key[1]);
  memcpy(out, r.v, sizeof(r.v));
}

static const uint32_t SALT_SPIN = 0x5350494eu, SALT_GAUSS = 0x47415553u, SALT_CAT = 0x43415400u;
static const uint32_t SALT_DENSE_SPIN = 0x44535049u, SALT_DENSE_GAUSS = 0x44474155u;
static const uint32_t SALT_LATTICE_SPIN = 0x4C535049u, SALT_LATTICE_REFILL = 0x4C524546u;
static const uint32_t SALT_LATTICE_PLANES = 0x4C504C30u;

static double or_uniform(uint32_t bits) { return (double)((((bits >> 9) << 1) | 1u)) * 5.9604644775390625e-08; }

/* the 23-bit bit-plane draw of rng layout 4, as the top 23 bits of a word: bit 22 - b is bit
 * 8 (row % 4) + (row % 32) / 4 of word b % 4 of counter (chain, row / 32, sweep, "LPL0" + b / 4) */
static uint32_t or_plane_bits(int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  const int s = (int)(row & 31), pos = 8 * (s & 3) + (s >> 2);
  uint32_t m = 0;
  or_u32x4 r = {{0, 0, 0, 0}};
  for (int b = 0; b < 23; ++b) {
    if ((b & 3) == 0)
      r = or_philox((uint32_t)gc, (uint32_t)(row >> 5), sweep, SALT_LATTICE_PLANES + (uint32_t)(b >> 2), k0, k1);
    m |= ((r.v[b & 3] >> pos) & 1u) << (22 - b);
  }
  return m << 9;
}

/* the 23-bit bit-plane draw of rng layout 5 ("planes8"), as the top 23 bits of a word: bit 22 - b
 * is bit 8 (row % 4) + chain % 8 of word b % 4 of counter (chain / 8, row / 4, sweep, "LPL0" + b / 4) */
static uint32_t or_plane8_bits(int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  const int pos = 8 * (int)(row & 3) + (int)(gc & 7);
  uint32_t m = 0;
  or_u32x4 r = {{0, 0, 0, 0}};
  for (int b = 0; b < 23; ++b) {
    if ((b & 3) == 0)
      r = or_philox((uint32_t)(gc >> 3), (uint32_t)(row >> 2), sweep, SALT_LATTICE_PLANES + (uint32_t)(b >> 2), k0,
                    k1);
    m |= ((r.v[b & 3] >> pos) & 1u) << (22 - b);
  }
  return m << 9;
}

/* the 23-bit split-uniform draw of rng layouts 2 and 3, as the top 23 bits of a word */
static uint32_t or_split_bits(int layout, int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  const int64_t pos = layout == 2 ? row : gc;
  const or_u32x4 r = layout == 2 ? or_philox((uint32_t)gc, (uint32_t)(row >> 3), sweep, SALT_LATTICE_SPIN, k0, k1)
                                 : or_philox((uint32_t)(gc >> 3), (uint32_t)row, sweep, SALT_LATTICE_SPIN, k0, k1);
  const uint32_t h = (r.v[(pos >> 1) & 3] >> (16 * (pos & 1))) & 0xFFFFu;
  const uint32_t f = or_philox((uint32_t)gc, (uint32_t)row, sweep, SALT_LATTICE_REFILL, k0, k1).v[0] >> 25;
  return ((h << 7) | f) << 9;
}

static double or_logit(double p) { return log(p) - log1p(-p); }

/* Categorical draw of the kernels' Philox mode, decided exactly: e_k =
 * exp(theta_k - max) in double, C_k = e_0 + ... + e_k, T_(k+1) = e_(k+1) +
 * ... (summed from the end), draw = number of k < q-1 with u >= C_k / S (the
 * inverse CDF of softmax(theta) at u).  margin: the smallest |logit(u) -
 * log(C_k / T_(k+1))| over the q-1 boundaries; the kernels' float32 decision
 * can differ from this one only inside the threshold band. */
static int or_categorical_icdf(const float* theta, int q, double u, double* margin) {
  double mx = theta[0];
  for (int k = 1; k < q; ++k) mx = fmax(mx, (double)theta[k]);
  double e[OR_MAXQ], head[OR_MAXQ], tail[OR_MAXQ + 1];
  double s = 0.0;
  for (int k = 0; k < q; ++k) {
    e[k] = exp((double)theta[k] - mx);
    s += e[k];
    head[k] = s;
  }
  tail[q] = 0.0;
  for (int k = q - 1; k >= 0; --k) tail[k] = tail[k + 1] + e[k];
  const double lu = or_logit(u);
  int cat = 0;
  double mg = INFINITY;
  for (int k = 0; k < q - 1; ++k) {
    const int reached = u < 0.5 ? head[k] <= u * s : (1.0 - u) * s <= tail[k + 1];
    cat += reached;
    if (head[k] > 0.0 && tail[k + 1] > 0.0) {
      const double d = fabs(lu - (log(head[k]) - log(tail[k + 1])));
      if (d < mg) mg = d;
    }
  }
  *margin = mg;
  return cat;
}

/* Philox-mode uniform of a spin draw at (global chain gc, flat row, sweep) in the kernel's counter layout
 * (see or_block.rng_layout). */
static double or_spin_uniform(int layout, int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  if (layout == 4) return or_uniform(or_plane_bits(gc, row, sweep, k0, k1));
  if (layout == 5) return or_uniform(or_plane8_bits(gc, row, sweep, k0, k1));
  if (layout == 2 || layout == 3) return or_uniform(or_split_bits(layout, gc, row, sweep, k0, k1));
  if (layout == 1) return or_uniform(or_philox((uint32_t)gc, (uint32_t)(row >> 2), sweep, SALT_DENSE_SPIN, k0, k1).v[row & 3]);
  return or_uniform(or_philox((uint32_t)(gc >> 2), (uint32_t)row, sweep, SALT_SPIN, k0, k1).v[gc & 3]);
}

/* Philox-mode standard normal of a gaussian draw: Box-Muller on two uniforms of one counter.  Generic
 * kernels: counter (chain, row, sweep, "GAUS"), words 0 and 1, the cosine output.  Dense kernel (layout 1):
 * counter (chain, row/4, sweep, "DGAU") serves four rows, words 2p and 2p+1 for rows 4j+2p and 4j+2p+1,
 * the cosine output for the even row and the sine output for the odd one. */
static double or_gauss_normal(int layout, int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  if (layout == 1) {
    const or_u32x4 r = or_philox((uint32_t)gc, (uint32_t)(row >> 2), sweep, SALT_DENSE_GAUSS, k0, k1);
    const int w = (int)((row >> 1) & 1) * 2;
    const double rad = sqrt(-2.0 * log(or_uniform(r.v[w]))), th = 2.0 * M_PI * or_uniform(r.v[w + 1]);
    return (row & 1) ? rad * sin(th) : rad * cos(th);
  }
  const or_u32x4 r = or_philox((uint32_t)gc, (uint32_t)row, sweep, SALT_GAUSS, k0, k1);
  return sqrt(-2.0 * log(or_uniform(r.v[0]))) * cos(2.0 * M_PI * or_uniform(r.v[1]));
}

/* Philox-mode uniform of a categorical draw: counter (chain/4, row, sweep), word chain % 4. */
static double or_cat_uniform(int64_t gc, int64_t row, uint32_t sweep, uint32_t k0, uint32_t k1) {
  return or_uniform(or_philox((uint32_t)(gc >> 2), (uint32_t)row, sweep, SALT_CAT, k0, k1).v[gc & 3]);
}

/* Gumbel-max over theta + g (first maximum), margin = best - second best (compiler.py:327-344). */
static int or_categorical_argmax(const float* theta, const float* g, int64_t g_stride, int q, double* margin) {
  int best = 0;
  double bv = 0.0, second = -INFINITY;
  for (int k = 0; k < q; ++k) {
    const double pk = (float)(theta[k] + g[k * g_stride]);
    if (k == 0 || pk > bv) {
      if (k) second = bv;
      bv = pk;
      best = k;
    } else if (pk > second) {
      second = pk;
    }
  }
  *margin = q > 1 ? bv - second : INFINITY;
  return best;
}

/* ---- field ---- */

static float st(const float* s, int64_t row, int64_t C, int64_t c) { return s[row * C + c]; }

/* selected weight offset of term e, -1 when a categorical value is out of range */
static int64_t cat_sel(const or_interaction* it, const float* s, int64_t C, int64_t c, int64_t e) {
  int64_t sel = 0;
  const int first = it->n_sources - it->n_categorical;
  for (int j = 0; j < it->n_categorical; ++j) {
    const float v = st(s, it->sources[(int64_t)(first + j) * it->nnz + e], C, c);
    const int q = it->cat_q[j];
    const int k = (int)v;
    if (!(v == (float)k) || k < 0 || k >= q) return -1;
    sel = sel * q + k;
  }
  return sel;
}

static float scale_of(const or_interaction* it, const float* s, int64_t C, int64_t c, int64_t e) {
  const int n_mult = it->n_sources - it->n_categorical;
  float p = st(s, it->sources[e], C, c);
  for (int j = 1; j < n_mult; ++j) p = p * st(s, it->sources[(int64_t)j * it->nnz + e], C, c);
  return p;
}

/* gamma over the interactions whose kind matches want_precision; *any = 0 when none */
static float scalar_field(const or_block* B, int want_precision, const float* s, int64_t C, int64_t c, int64_t i,
                          int* any) {
  float gamma = 0.0f;
  *any = 0;
  for (int k = 0; k < B->n_interactions; ++k) {
    const or_interaction* it = &B->inter[k];
    if ((it->kind == OR_KIND_PRECISION) != (want_precision != 0)) continue;
    const int n_mult = it->n_sources - it->n_categorical;
    float contrib = 0.0f;
    int first = 1;
    for (int64_t e = it->row_ptr[i]; e < it->row_ptr[i + 1]; ++e) {
      float w;
      if (it->n_categorical) {
        const int64_t sel = cat_sel(it, s, C, c, e);
        w = sel < 0 ? 0.0f : it->weights[e * it->w_inner + sel];
      } else {
        w = it->weights[e * it->w_inner];
      }
      float term = n_mult ? w * scale_of(it, s, C, c, e) : w;
      contrib = first ? term : contrib + term;
      first = 0;
    }
    gamma = *any ? gamma + contrib : contrib;
    *any = 1;
  }
  return gamma;
}

static void theta_of(const or_block* B, const float* s, int64_t C, int64_t c, int64_t i, float* theta) {
  const int q = B->q;
  int seen = 0;
  for (int k = 0; k < q; ++k) theta[k] = 0.0f;
  for (int n = 0; n < B->n_interactions; ++n) {
    const or_interaction* it = &B->inter[n];
    const int n_mult = it->n_sources - it->n_categorical;
    const int64_t cat_prod = it->w_inner / q;
    float contrib[OR_MAXQ];
    for (int k = 0; k < q; ++k) contrib[k] = 0.0f;
    int first = 1;
    for (int64_t e = it->row_ptr[i]; e < it->row_ptr[i + 1]; ++e) {
      const int64_t sel = it->n_categorical ? cat_sel(it, s, C, c, e) : 0;
      const float scale = n_mult ? scale_of(it, s, C, c, e) : 1.0f;
      for (int k = 0; k < q; ++k) {
        const float w = sel < 0 ? 0.0f : it->weights[e * it->w_inner + k * cat_prod + sel];
        float term = n_mult ? w * scale : w;
        float acc = first ? term : contrib[k] + term;
        contrib[k] = acc;
      }
      first = 0;
    }
    for (int k = 0; k < q; ++k) {
      float t = seen ? theta[k] + contrib[k] : contrib[k];
      theta[k] = t;
    }
    seen = 1;
  }
}

typedef struct {
  const or_block* B;
  const float* state;
  float* out;
  double* margin;
  int64_t C, chain_offset, base, i0, i1;
  int32_t use_variates;
  uint32_t sweep, k0, k1;
} or_task;

static void* run_rows(void* arg) {
  const or_task* t = (const or_task*)arg;
  const or_block* B = t->B;
  const float* state = t->state;
  const int64_t C = t->C;
  for (int64_t i = t->i0; i < t->i1; ++i) {
    const int64_t row = B->row_start + i;
    for (int64_t c = 0; c < C; ++c) {
      const int64_t gc = t->chain_offset + c;
      const int64_t o = (t->base + i) * C + c;
      double m = 0.0;
      float v;
      if (B->family == OR_SPIN) {
        int any;
        const float gamma = scalar_field(B, 0, state, C, c, i, &any);
        const float two_g = 2.0f * gamma;
        if (t->use_variates) {
          const float l = B->variates[i * C + c];
          v = two_g > l ? 1.0f : -1.0f;
          m = (double)two_g - (double)l;
        } else {
          const double u = or_spin_uniform(B->rng_layout, gc, row, t->sweep, t->k0, t->k1);
          const double l = log(u) - log1p(-u);
          m = (double)two_g - l;
          v = m > 0.0 ? 1.0f : -1.0f;
        }
      } else if (B->family == OR_CATEGORICAL) {
        float theta[OR_MAXQ];
        theta_of(B, state, C, c, i, theta);
        const int q = B->q;
        if (t->use_variates) {
          v = (float)or_categorical_argmax(theta, B->variates + (int64_t)i * q * C + c, C, q, &m);
        } else {
          v = (float)or_categorical_icdf(theta, q, or_cat_uniform(gc, row, t->sweep, t->k0, t->k1), &m);
        }
      } else {
        int any_l, any_p;
        const float lin = scalar_field(B, 0, state, C, c, i, &any_l);
        float prec = scalar_field(B, 1, state, C, c, i, &any_p);
        if (!any_p) prec = 1.0f;
        const float linear = any_l ? lin : 0.0f;
        const float pe = prec + 1e-6f;
        const float inv = 1.0f / pe;
        const float mean = linear * inv;
        const float sd = sqrtf(inv);
        if (t->use_variates) {
          const float tt = sd * B->variates[i * C + c];
          v = mean + tt;
        } else {
          const double xi = or_gauss_normal(B->rng_layout, gc, row, t->sweep, t->k0, t->k1);
          v = (float)((double)mean + (double)sd * xi);
        }
      }
      t->out[o] = v;
      if (t->margin) t->margin[o] = m;
    }
  }
  return NULL;
}

/*
 * One group step.  state: [rows][C] float32, updated in place after all
 * blocks are sampled.  margin (optional): [sum n_nodes][C] distance to the
 * decision boundary (spin: 2*gamma - l; categorical: best - second best;
 * gaussian: 0).  n_threads host threads split each block's rows.  Returns 0,
 * or -1 when memory runs out.
 */
int oracle_group_step(const or_block* blocks, int32_t n_blocks, float* state, int64_t C, int64_t chain_offset,
                      int32_t use_variates, uint64_t seed, uint32_t sweep, double* margin, int32_t n_threads) {
  int64_t rows = 0;
  for (int b = 0; b < n_blocks; ++b) rows += blocks[b].n_nodes;
  float* out = (float*)malloc(sizeof(float) * (size_t)(rows > 0 ? rows : 1) * (size_t)C);
  if (!out) return -1;
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  pthread_t th[256];
  or_task tasks[256];
  int64_t base = 0;
  for (int b = 0; b < n_blocks; ++b) {
    const int64_t n = blocks[b].n_nodes;
    const int nt = (int)(n < n_threads ? (n > 0 ? n : 1) : n_threads);
    for (int k = 0; k < nt; ++k) {
      or_task* t = &tasks[k];
      t->B = &blocks[b];
      t->state = state;
      t->out = out;
      t->margin = margin;
      t->C = C;
      t->chain_offset = chain_offset;
      t->base = base;
      t->i0 = n * k / nt;
      t->i1 = n * (k + 1) / nt;
      t->use_variates = use_variates;
      t->sweep = sweep;
      t->k0 = (uint32_t)seed;
      t->k1 = (uint32_t)(seed >> 32);
    }
    int started = 0;
    for (int k = 1; k < nt; ++k) {
      if (pthread_create(&th[k], NULL, run_rows, &tasks[k]) != 0) break;
      started = k;
    }
    run_rows(&tasks[0]);
    for (int k = 1; k <= started; ++k) pthread_join(th[k], NULL);
    for (int k = started + 1; k < nt; ++k) run_rows(&tasks[k]);
    base += n;
  }
  base = 0;
  for (int b = 0; b < n_blocks; ++b) {
    const or_block* B = &blocks[b];
    memcpy(state + B->row_start * C, out + base * C, sizeof(float) * (size_t)(B->n_nodes * C));
    base += B->n_nodes;
  }
  free(out);
  return 0;
}

int oracle_abi_version(void) { return 1; }

/* ======================================================================
 * Model paths without per-term tables.  Each restates, for one model family
 * built from its raw parameters, the same group math as the table path above
 * (the tests check both paths against each other on small models), so the
 * configurations too large for per-term tables are checked at full size.
 * ====================================================================== */

/* Runs fn(arg, i0, i1) over [0, n) split across n_threads threads. */
typedef struct {
  void (*fn)(const void*, int64_t, int64_t);
  const void* arg;
  int64_t i0, i1;
} or_span;

static void* or_span_main(void* p) {
  const or_span* s = (const or_span*)p;
  s->fn(s->arg, s->i0, s->i1);
  return NULL;
}

static void or_parallel(void (*fn)(const void*, int64_t, int64_t), const void* arg, int64_t n, int n_threads) {
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  if (n < n_threads) n_threads = (int)(n > 0 ? n : 1);
  pthread_t th[256];
  or_span sp[256];
  for (int k = 0; k < n_threads; ++k) {
    sp[k].fn = fn;
    sp[k].arg = arg;
    sp[k].i0 = n * k / n_threads;
    sp[k].i1 = n * (k + 1) / n_threads;
  }
  int started = 0;
  for (int k = 1; k < n_threads; ++k) {
    if (pthread_create(&th[k], NULL, or_span_main, &sp[k]) != 0) break;
    started = k;
  }
  or_span_main(&sp[0]);
  for (int k = 1; k <= started; ++k) pthread_join(th[k], NULL);
  for (int k = started + 1; k < n_threads; ++k) or_span_main(&sp[k]);
}

/* ---- 2-D Ising lattice ----
 * Periodic height x width lattice (both even), site (y, x) at L = y*width + x
 * with colour (x + y) % 2.  Block c holds the colour-c sites in increasing L,
 * so site L sits at block row L / 2 and flat row c*n/2 + L/2.  A site's field
 * is the bias interaction followed by the pair interaction over its
 * neighbours in the order (left, right, up, down), each term weight x spin:
 *   gamma = b + (((w*s_l + w*s_r) + w*s_u) + w*s_d)
 * in float32 (w = beta*J, b = beta*h), the order the table path sums the
 * lattice's per-edge tables in. */
typedef struct {
  int64_t height, width;
  float edge_weight, site_bias;
} or_lattice2d;

typedef struct {
  const or_lattice2d* L;
  int32_t colour, rng_layout, use_variates;
  float* state;
  const float* variates;
  double* margin;
  int64_t C, chain_offset;
  uint32_t sweep, k0, k1;
} or_ising_task;

static void or_ising_rows(const void* arg, int64_t r0, int64_t r1) {
  const or_ising_task* t = (const or_ising_task*)arg;
  const int64_t H = t->L->height, W = t->L->width, half = H * W / 2, C = t->C;
  const float w = t->L->edge_weight, b = t->L->site_bias;
  const int64_t own0 = (int64_t)t->colour * half, oth0 = (int64_t)(1 - t->colour) * half;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t y = (2 * r) / W;
    const int64_t x = (2 * r) % W + ((y + t->colour) & 1);
    const int64_t nb[4] = {y * W + (x + W - 1) % W, y * W + (x + 1) % W, ((y + H - 1) % H) * W + x,
                           ((y + 1) % H) * W + x};
    const int64_t row = own0 + r;
    for (int64_t c = 0; c < C; ++c) {
      float acc = w * t->state[(oth0 + nb[0] / 2) * C + c];
      for (int k = 1; k < 4; ++k) {
        const float term = w * t->state[(oth0 + nb[k] / 2) * C + c];
        acc = acc + term;
      }
      const float gamma = b + acc;
      const float two_g = 2.0f * gamma;
      double m;
      if (t->use_variates) {
        const float lf = t->variates[r * C + c];
        m = (double)two_g - (double)lf;
        t->state[row * C + c] = two_g > lf ? 1.0f : -1.0f;
      } else {
        const double u = or_spin_uniform(t->rng_layout, t->chain_offset + c, row, t->sweep, t->k0, t->k1);
        m = (double)two_g - (log(u) - log1p(-u));
        t->state[row * C + c] = m > 0.0 ? 1.0f : -1.0f;
      }
      if (t->margin) t->margin[r * C + c] = m;
    }
  }
}

/* One colour half-sweep of the lattice on the float32 state [n][C] (block rows as above).  The colour's
 * sites read only the other colour, so they are written in place.  variates: [n/2][C] logits or NULL
 * (Philox, rng_layout as in or_block).  margin: [n/2][C] or NULL. */
int oracle_ising2d_step(const or_lattice2d* L, int32_t colour, float* state, int64_t C, int64_t chain_offset,
                        const float* variates, int32_t rng_layout, uint64_t seed, uint32_t sweep, double* margin,
                        int32_t n_threads) {
  if (!L || L->height % 2 || L->width % 2 || L->height <= 0 || L->width <= 0 || (colour & ~1)) return -1;
  or_ising_task t = {L, colour, rng_layout, variates != NULL, state, variates, margin, C, chain_offset, sweep,
                     (uint32_t)seed, (uint32_t)(seed >> 32)};
  or_parallel(or_ising_rows, &t, L->height * L->width / 2, n_threads);
  return 0;
}

/* ---- 3-D Potts lattice ----
 * Periodic X x Y x Z lattice (all even), site (x, y, z) at L = (z*Y + y)*X + x
 * with colour (x + y + z) % 2, block c = colour-c sites in increasing L, block
 * row L / 2.  Field of category k: the bias interaction, then per axis a in
 * (x, y, z) the pair interaction over the two neighbours (minus, plus), each
 * term selecting J[a][k][s_neighbour]:
 *   theta_k = ((b_k + (Jx[k][s_x-] + Jx[k][s_x+])) + (Jy[k][s_y-] + Jy[k][s_y+]))
 *             + (Jz[k][s_z-] + Jz[k][s_z+])
 * in float32.  A neighbour category outside [0, q) selects weight 0. */
typedef struct {
  int64_t dims[3];
  int32_t q;
  const float* J;      /* [3][q][q] */
  const float* bias0;  /* [n/2][q], block 0 in row order */
  const float* bias1;  /* [n/2][q], block 1 */
} or_potts3d;

typedef struct {
  const or_potts3d* P;
  int32_t colour, use_variates;
  float* state;
  const float* variates;
  double* margin;
  int64_t C, chain_offset;
  uint32_t sweep, k0, k1;
} or_potts_task;

static void or_potts_rows(const void* arg, int64_t r0, int64_t r1) {
  const or_potts_task* t = (const or_potts_task*)arg;
  const int64_t X = t->P->dims[0], Y = t->P->dims[1], Z = t->P->dims[2], half = X * Y * Z / 2, C = t->C;
  const int q = t->P->q;
  const float* bias = t->colour ? t->P->bias1 : t->P->bias0;
  const int64_t own0 = (int64_t)t->colour * half, oth0 = (int64_t)(1 - t->colour) * half;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t even = 2 * r;
    const int64_t y0 = (even / X) % Y, z = even / (X * Y);
    const int64_t Ls = even + ((y0 + z + t->colour) & 1);
    const int64_t x = Ls % X, y = (Ls / X) % Y;
    int64_t nb[6];
    nb[0] = (z * Y + y) * X + (x + X - 1) % X;
    nb[1] = (z * Y + y) * X + (x + 1) % X;
    nb[2] = (z * Y + (y + Y - 1) % Y) * X + x;
    nb[3] = (z * Y + (y + 1) % Y) * X + x;
    nb[4] = (((z + Z - 1) % Z) * Y + y) * X + x;
    nb[5] = (((z + 1) % Z) * Y + y) * X + x;
    const int64_t row = own0 + r;
    for (int64_t c = 0; c < C; ++c) {
      int sn[6];
      for (int j = 0; j < 6; ++j) {
        const float v = t->state[(oth0 + nb[j] / 2) * C + c];
        const int k = (int)v;
        sn[j] = (v == (float)k && k >= 0 && k < q) ? k : -1;
      }
      float theta[OR_MAXQ];
      for (int k = 0; k < q; ++k) {
        float acc = bias[r * q + k];
        for (int a = 0; a < 3; ++a) {
          const float* Ja = t->P->J + (int64_t)a * q * q + (int64_t)k * q;
          const float lo = sn[2 * a] < 0 ? 0.0f : Ja[sn[2 * a]];
          const float hi = sn[2 * a + 1] < 0 ? 0.0f : Ja[sn[2 * a + 1]];
          const float pair = lo + hi;
          acc = acc + pair;
        }
        theta[k] = acc;
      }
      double m;
      int cat;
      if (t->use_variates) {
        cat = or_categorical_argmax(theta, t->variates + r * q * C + c, C, q, &m);
      } else {
        cat = or_categorical_icdf(theta, q, or_cat_uniform(t->chain_offset + c, row, t->sweep, t->k0, t->k1), &m);
      }
      t->state[row * C + c] = (float)cat;
      if (t->margin) t->margin[r * C + c] = m;
    }
  }
}

/* One colour half-sweep of the Potts lattice on the float32 state [n][C] (categories as floats), in place.
 * variates: [n/2][q][C] Gumbel noise or NULL (Philox, chain4 counters, inverse-CDF draw). */
int oracle_potts3d_step(const or_potts3d* P, int32_t colour, float* state, int64_t C, int64_t chain_offset,
                        const float* variates, uint64_t seed, uint32_t sweep, double* margin, int32_t n_threads) {
  if (!P || P->q < 1 || P->q > OR_MAXQ || (colour & ~1)) return -1;
  for (int a = 0; a < 3; ++a)
    if (P->dims[a] <= 0 || P->dims[a] % 2) return -1;
  or_potts_task t = {P, colour, variates != NULL, state, variates, margin, C, chain_offset, sweep, (uint32_t)seed,
                     (uint32_t)(seed >> 32)};
  or_parallel(or_potts_rows, &t, P->dims[0] * P->dims[1] * P->dims[2] / 2, n_threads);
  return 0;
}

/* ---- dense bipartite (restricted Boltzmann machine) ----
 * Visible block rows [0, V), hidden block rows [V, V + H).  Field of hidden
 * unit j: b_h[j] + sum_i W[i][j] v_i; of visible unit i: b_v[i] + sum_j
 * W[i][j] h_j.  The fields are summed in double precision: the exact value
 * every float32 summation order approximates, so a kernel's decision can be
 * judged against it with the threshold band (its float32 rounding, about
 * 1e-6 at these sizes, is well inside 1e-5).  Spin units: +1 where 2*gamma >
 * logit(u); gaussian units (precision 1, the reference's default): mean =
 * gamma / (1 + 1e-6), sd = sqrt(1 / (1 + 1e-6)), value = mean + sd * xi,
 * rounded to bfloat16 (nearest even) when store_bf16 is set (the kernels'
 * bf16 operand storage). */
typedef struct {
  int64_t n_visible, n_hidden;
  const float* W;   /* [V][H] */
  const float* b_v; /* [V] */
  const float* b_h; /* [H] */
  int32_t visible_family, store_bf16;
} or_dense;

typedef struct {
  const or_dense* D;
  int32_t block, family, rng_layout, use_variates;
  float* state;
  const float* variates;
  double* margin;
  float* out;
  int64_t C, chain_offset;
  uint32_t sweep, k0, k1;
} or_dense_task;

static float or_bf16_round(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  if ((b & 0x7F800000u) == 0x7F800000u) return x; /* inf / nan */
  b = (b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u;
  float y;
  memcpy(&y, &b, 4);
  return y;
}

#define OR_DENSE_TILE 32

static void or_dense_units(const void* arg, int64_t t0, int64_t t1) {
  const or_dense_task* t = (const or_dense_task*)arg;
  const int64_t V = t->D->n_visible, Hh = t->D->n_hidden, C = t->C;
  const int hidden = t->block == 1;
  const int64_t n_units = hidden ? Hh : V, n_src = hidden ? V : Hh;
  const int64_t src0 = hidden ? 0 : V, row0 = hidden ? V : 0;
  const float* bias = hidden ? t->D->b_h : t->D->b_v;
  double* acc = (double*)malloc(sizeof(double) * OR_DENSE_TILE * (size_t)C);
  if (!acc) return;
  for (int64_t tile = t0; tile < t1; ++tile) {
    const int64_t u0 = tile * OR_DENSE_TILE;
    const int64_t nu = n_units - u0 < OR_DENSE_TILE ? n_units - u0 : OR_DENSE_TILE;
    for (int64_t a = 0; a < nu; ++a)
      for (int64_t c = 0; c < C; ++c) acc[a * C + c] = bias[u0 + a];
    for (int64_t s = 0; s < n_src; ++s) {
      const float* src = t->state + (src0 + s) * C;
      for (int64_t a = 0; a < nu; ++a) {
        const double w = hidden ? t->D->W[s * Hh + u0 + a] : t->D->W[(u0 + a) * Hh + s];
        double* ac = acc + a * C;
        for (int64_t c = 0; c < C; ++c) ac[c] += w * (double)src[c];
      }
    }
    for (int64_t a = 0; a < nu; ++a) {
      const int64_t unit = u0 + a, row = row0 + unit;
      for (int64_t c = 0; c < C; ++c) {
        const double gamma = acc[a * C + c];
        const int64_t gc = t->chain_offset + c;
        double m = 0.0;
        float v;
        if (t->family == OR_SPIN) {
          double l;
          if (t->use_variates) {
            l = t->variates[unit * C + c];
          } else {
            const double u = or_spin_uniform(t->rng_layout, gc, row, t->sweep, t->k0, t->k1);
            l = log(u) - log1p(-u);
          }
          m = 2.0 * gamma - l;
          v = m > 0.0 ? 1.0f : -1.0f;
        } else {
          const float pe = 1.0f + 1e-6f;
          const float inv = 1.0f / pe;
          const double xi = t->use_variates ? (double)t->variates[unit * C + c]
                                            : or_gauss_normal(t->rng_layout, gc, row, t->sweep, t->k0, t->k1);
          v = (float)(gamma * (double)inv + (double)sqrtf(inv) * xi);
          if (t->D->store_bf16) v = or_bf16_round(v);
        }
        t->out[unit * C + c] = v;
        if (t->margin) t->margin[unit * C + c] = m;
      }
    }
  }
  free(acc);
}

/* Samples one block (0 visible, 1 hidden) of the dense bipartite model on the float32 state [V+H][C] and
 * writes it in place (the block reads only the other block).  variates: [n_units][C] (spin logits or
 * standard normals) or NULL (Philox, rng_layout as in or_block).  margin: [n_units][C] or NULL. */
int oracle_dense_step(const or_dense* D, int32_t block, float* state, int64_t C, int64_t chain_offset,
                      const float* variates, int32_t rng_layout, uint64_t seed, uint32_t sweep, double* margin,
                      int32_t n_threads) {
  if (!D || (block & ~1)) return -1;
  const int64_t n_units = block ? D->n_hidden : D->n_visible;
  float* out = (float*)malloc(sizeof(float) * (size_t)(n_units > 0 ? n_units : 1) * (size_t)C);
  if (!out) return -1;
  or_dense_task t = {D, block, block ? OR_SPIN : D->visible_family, rng_layout, variates != NULL, state, variates,
                     margin, out, C, chain_offset, sweep, (uint32_t)seed, (uint32_t)(seed >> 32)};
  or_parallel(or_dense_units, &t, (n_units + OR_DENSE_TILE - 1) / OR_DENSE_TILE, n_threads);
  memcpy(state + (block ? D->n_visible : 0) * C, out, sizeof(float) * (size_t)(n_units * C));
  free(out);
  return 0;
}

/* ---- greedy colouring ----
 * Nodes in index order; each takes the smallest colour that none of its
 * already-coloured neighbours has (the colouring that defines the sparse
 * random-graph configuration's blocks).  colour: [n]; *n_colours = k. */
int oracle_greedy_colouring(int64_t n, const int64_t* row_ptr, const int32_t* cols, int32_t* colour,
                            int32_t* n_colours) {
  int64_t cap = 64;
  int64_t* seen = (int64_t*)malloc(sizeof(int64_t) * (size_t)cap); /* seen[k] == v: colour k is next to v */
  if (!seen) return -1;
  for (int64_t k = 0; k < cap; ++k) seen[k] = -1;
  int32_t k_max = 0;
  for (int64_t v = 0; v < n; ++v) {
    int64_t deg = row_ptr[v + 1] - row_ptr[v];
    if (deg + 1 > cap) {
      int64_t nc = cap;
      while (nc < deg + 1) nc *= 2;
      int64_t* ns = (int64_t*)realloc(seen, sizeof(int64_t) * (size_t)nc);
      if (!ns) {
        free(seen);
        return -1;
      }
      for (int64_t k = cap; k < nc; ++k) ns[k] = -1;
      seen = ns;
      cap = nc;
    }
    for (int64_t e = row_ptr[v]; e < row_ptr[v + 1]; ++e) {
      const int64_t u = cols[e];
      if (u < v && colour[u] < cap) seen[colour[u]] = v; /* lower-indexed neighbours are coloured */
    }
    int32_t k = 0;
    while (seen[k] == v) ++k;
    colour[v] = k;
    if (k + 1 > k_max) k_max = k + 1;
  }
  free(seen);
  *n_colours = k_max;
  return 0;
}
