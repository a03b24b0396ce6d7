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
          const int dense = B->rng_layout == 1;
          double u;
          if (B->rng_layout == 4) {
            u = or_uniform(or_plane_bits(gc, row, t->sweep, t->k0, t->k1));
          } else if (B->rng_layout == 5) {
            u = or_uniform(or_plane8_bits(gc, row, t->sweep, t->k0, t->k1));
          } else if (B->rng_layout == 2 || B->rng_layout == 3) {
            u = or_uniform(or_split_bits(B->rng_layout, gc, row, t->sweep, t->k0, t->k1));
          } else {
            const or_u32x4 r = dense ? or_philox((uint32_t)gc, (uint32_t)(row >> 2), t->sweep, SALT_DENSE_SPIN, t->k0, t->k1)
                                     : or_philox((uint32_t)(gc >> 2), (uint32_t)row, t->sweep, SALT_SPIN, t->k0, t->k1);
            u = or_uniform(r.v[dense ? (row & 3) : (gc & 3)]);
          }
          const double l = log(u) - log1p(-u);
          m = (double)two_g - l;
          v = m > 0.0 ? 1.0f : -1.0f;
        }
      } else if (B->family == OR_CATEGORICAL) {
        float theta[OR_MAXQ];
        theta_of(B, state, C, c, i, theta);
        const int q = B->q;
        if (t->use_variates) {
          int best = 0;
          double bv = 0.0, second = -INFINITY;
          for (int k = 0; k < q; ++k) {
            const double pk = (float)(theta[k] + B->variates[((int64_t)i * q + k) * C + c]);
            if (k == 0 || pk > bv) {
              if (k) second = bv;
              bv = pk;
              best = k;
            } else if (pk > second) {
              second = pk;
            }
          }
          v = (float)best;
          m = q > 1 ? bv - second : INFINITY;
        } else {
          const or_u32x4 r = or_philox((uint32_t)(gc >> 2), (uint32_t)row, t->sweep, SALT_CAT, t->k0, t->k1);
          v = (float)or_categorical_icdf(theta, q, or_uniform(r.v[gc & 3]), &m);
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
          const int dense = B->rng_layout == 1;
          const or_u32x4 r = dense ? or_philox((uint32_t)gc, (uint32_t)(row >> 1), t->sweep, SALT_DENSE_GAUSS, t->k0, t->k1)
                                   : or_philox((uint32_t)gc, (uint32_t)row, t->sweep, SALT_GAUSS, t->k0, t->k1);
          const int w = dense ? (int)(row & 1) * 2 : 0;
          const double xi = sqrt(-2.0 * log(or_uniform(r.v[w]))) * cos(2.0 * M_PI * or_uniform(r.v[w + 1]));
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
