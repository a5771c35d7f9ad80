/*
 * C float64 restatement of the reference's test oracle.
 *
 * TEST INFRASTRUCTURE ONLY. This library is a checker and the timed CPU baseline: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline legs may load it. The product path never
 * routes through it.
 *
 * It restates tests/support/reference.rs (the reference's straight-line float64 forward of one
 * image; the Rust crate cannot be built here: no cargo/rustc, and its runtime hrx-rs is not
 * vendored). Citations are to that file unless another file is named. Third-party arithmetic:
 * matrixmultiply 0.3.11 `dgemm` (Cargo.lock:1479-1481) is restated as a plain blocked float64
 * GEMM that accumulates every output element in ascending-k order.
 *
 * Pinned by tests/golden/ (Hugging Face transformers DINOv3ViTModel run in float64 on the
 * same seeded weights and images) and cross-checked against oracle/ref_numpy.py.
 *
 * Threads: ref_forward parallelises over images with OpenMP (the reference is single-threaded
 * per image: matrixmultiply's `threading` feature is off, Cargo.toml:22-24).
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define T 201
#define H 384
#define HEADS 6
#define HD 64
#define MLPH 1536
#define NLAYERS 12
#define PREFIX 5

typedef struct {
  double *norm1_w, *norm1_b, *norm2_w, *norm2_b;
  double *qT, *kT, *vT, *oT; /* transposed [k][n] */
  double *q_b, *v_b, *o_b, *ls1, *ls2;
  double *gateT, *upT, *downT, *gate_b, *up_b, *down_b;
} ref_layer;

typedef struct ref_model {
  double *patchT; /* [768][384] */
  double *patch_b, *cls, *regs, *norm_w, *norm_b;
  ref_layer layer[NLAYERS];
  int have; /* number of tensors set */
} ref_model;

ref_model *ref_model_new(void) { return (ref_model *)calloc(1, sizeof(ref_model)); }

static void free_if(double *p) { free(p); }

void ref_model_free(ref_model *m) {
  if (!m) return;
  free_if(m->patchT); free_if(m->patch_b); free_if(m->cls); free_if(m->regs);
  free_if(m->norm_w); free_if(m->norm_b);
  for (int i = 0; i < NLAYERS; i++) {
    ref_layer *l = &m->layer[i];
    double *all[] = {l->norm1_w, l->norm1_b, l->norm2_w, l->norm2_b, l->qT, l->kT, l->vT, l->oT,
                     l->q_b, l->v_b, l->o_b, l->ls1, l->ls2, l->gateT, l->upT, l->downT,
                     l->gate_b, l->up_b, l->down_b};
    for (size_t j = 0; j < sizeof(all) / sizeof(all[0]); j++) free_if(all[j]);
  }
  free(m);
}

static double *copy_vec(const float *src, size_t n) {
  double *d = (double *)malloc(n * sizeof(double));
  for (size_t i = 0; i < n; i++) d[i] = (double)src[i];
  return d;
}

/* W is [n][k] (PyTorch Linear layout); store it as [k][n] so the GEMM streams rows. */
static double *copy_transposed(const float *src, int n, int k) {
  double *d = (double *)malloc((size_t)n * k * sizeof(double));
  for (int r = 0; r < n; r++)
    for (int c = 0; c < k; c++) d[(size_t)c * n + r] = (double)src[(size_t)r * k + c];
  return d;
}

/* Returns 0 when the name is known and the size matches, -1 otherwise. */
int ref_model_set(ref_model *m, const char *name, const float *data, size_t n) {
#define VEC(field, want)                                    \
  do {                                                      \
    if (n != (size_t)(want)) return -1;                     \
    free(field); field = copy_vec(data, n); m->have++;      \
    return 0;                                               \
  } while (0)
#define MAT(field, rows, cols)                                  \
  do {                                                          \
    if (n != (size_t)(rows) * (cols)) return -1;                \
    free(field); field = copy_transposed(data, rows, cols); m->have++; \
    return 0;                                                   \
  } while (0)
  if (!strcmp(name, "embeddings.patch_embeddings.weight")) MAT(m->patchT, H, 768);
  if (!strcmp(name, "embeddings.patch_embeddings.bias")) VEC(m->patch_b, H);
  if (!strcmp(name, "embeddings.cls_token")) VEC(m->cls, H);
  if (!strcmp(name, "embeddings.register_tokens")) VEC(m->regs, 4 * H);
  if (!strcmp(name, "norm.weight")) VEC(m->norm_w, H);
  if (!strcmp(name, "norm.bias")) VEC(m->norm_b, H);
  int li = -1, off = 0;
  if (strncmp(name, "layer.", 6) == 0) {
    li = atoi(name + 6);
    const char *dot = strchr(name + 6, '.');
    if (!dot || li < 0 || li >= NLAYERS) return -1;
    off = (int)(dot - name) + 1;
  } else {
    return -1;
  }
  const char *s = name + off;
  ref_layer *l = &m->layer[li];
  if (!strcmp(s, "norm1.weight")) VEC(l->norm1_w, H);
  if (!strcmp(s, "norm1.bias")) VEC(l->norm1_b, H);
  if (!strcmp(s, "norm2.weight")) VEC(l->norm2_w, H);
  if (!strcmp(s, "norm2.bias")) VEC(l->norm2_b, H);
  if (!strcmp(s, "attention.q_proj.weight")) MAT(l->qT, H, H);
  if (!strcmp(s, "attention.k_proj.weight")) MAT(l->kT, H, H);
  if (!strcmp(s, "attention.v_proj.weight")) MAT(l->vT, H, H);
  if (!strcmp(s, "attention.o_proj.weight")) MAT(l->oT, H, H);
  if (!strcmp(s, "attention.q_proj.bias")) VEC(l->q_b, H);
  if (!strcmp(s, "attention.v_proj.bias")) VEC(l->v_b, H);
  if (!strcmp(s, "attention.o_proj.bias")) VEC(l->o_b, H);
  if (!strcmp(s, "layer_scale1.lambda1")) VEC(l->ls1, H);
  if (!strcmp(s, "layer_scale2.lambda1")) VEC(l->ls2, H);
  if (!strcmp(s, "mlp.gate_proj.weight")) MAT(l->gateT, MLPH, H);
  if (!strcmp(s, "mlp.up_proj.weight")) MAT(l->upT, MLPH, H);
  if (!strcmp(s, "mlp.down_proj.weight")) MAT(l->downT, H, MLPH);
  if (!strcmp(s, "mlp.gate_proj.bias")) VEC(l->gate_b, MLPH);
  if (!strcmp(s, "mlp.up_proj.bias")) VEC(l->up_b, MLPH);
  if (!strcmp(s, "mlp.down_proj.bias")) VEC(l->down_b, H);
  return -1;
#undef VEC
#undef MAT
}

/* Tensors the forward needs: 6 globals + 19 per layer. */
int ref_model_missing(const ref_model *m) { return 6 + 19 * NLAYERS - m->have; }

/* out[m][n] = x[m][k] . W[n][k] + bias[n]  (reference.rs:5-37). wT is [k][n]. */
static void linear(const double *x, int rows, int k, const double *wT, int n, const double *bias,
                   double *out) {
  memset(out, 0, (size_t)rows * n * sizeof(double));
  const int MB = 8, NB = 512;
  for (int n0 = 0; n0 < n; n0 += NB) {
    int n1 = n0 + NB < n ? n0 + NB : n;
    for (int m0 = 0; m0 < rows; m0 += MB) {
      int m1 = m0 + MB < rows ? m0 + MB : rows;
      for (int kk = 0; kk < k; kk++) {
        const double *wr = wT + (size_t)kk * n;
        for (int i = m0; i < m1; i++) {
          double a = x[(size_t)i * k + kk];
          double *o = out + (size_t)i * n;
          for (int j = n0; j < n1; j++) o[j] += a * wr[j];
        }
      }
    }
  }
  if (bias)
    for (int i = 0; i < rows; i++)
      for (int j = 0; j < n; j++) out[(size_t)i * n + j] += bias[j];
}

/* LayerNorm, eps 1e-5, two-pass divide-by-H variance (reference.rs:38-48). */
static void norm(const double *x, const double *w, const double *b, double *out) {
  for (int r = 0; r < T; r++) {
    const double *s = x + (size_t)r * H;
    double mean = 0, var = 0;
    for (int c = 0; c < H; c++) mean += s[c];
    mean /= H;
    for (int c = 0; c < H; c++) var += (s[c] - mean) * (s[c] - mean);
    var /= H;
    double d = sqrt(var + 1e-5);
    for (int c = 0; c < H; c++) out[(size_t)r * H + c] = (s[c] - mean) / d * w[c] + b[c];
  }
}

/* [3][224][224] -> [196][768], inner order (c, dy, dx) (reference.rs:67-79). */
void ref_patchify(const float *image, double *patches) {
  size_t i = 0;
  for (int y = 0; y < 14; y++)
    for (int x = 0; x < 14; x++)
      for (int c = 0; c < 3; c++)
        for (int dy = 0; dy < 16; dy++)
          for (int dx = 0; dx < 16; dx++)
            patches[i++] = image[(size_t)c * 224 * 224 + (size_t)(y * 16 + dy) * 224 + x * 16 + dx];
}

/* cos/sin [196][64] exactly as the rotation uses them (reference.rs:112-118). */
void ref_rope_tables(double *cosv, double *sinv) {
  for (int patch = 0; patch < 196; patch++)
    for (int c = 0; c < 64; c++) {
      int pos = (c % 32 < 16) ? patch / 14 : patch % 14;
      double angle = 2.0 * M_PI * (2.0 * (pos + 0.5) / 14.0 - 1.0) / pow(100.0, (c % 16) / 16.0);
      cosv[patch * 64 + c] = cos(angle);
      sinv[patch * 64 + c] = sin(angle);
    }
}

typedef struct {
  double *x, *h, *q, *k, *v, *ctx, *tmp, *gate, *up, *patches, *scores, *cosv, *sinv, *orig;
} scratch;

static void forward_one(const ref_model *m, const float *image, double *out, scratch *s) {
  ref_patchify(image, s->patches);
  /* x = [cls; registers; patch_embed(patches)]  (reference.rs:80-88) */
  memcpy(s->x, m->cls, H * sizeof(double));
  memcpy(s->x + H, m->regs, 4 * H * sizeof(double));
  linear(s->patches, 196, 768, m->patchT, H, m->patch_b, s->x + PREFIX * H);
  for (int li = 0; li < NLAYERS; li++) {
    const ref_layer *l = &m->layer[li];
    norm(s->x, l->norm1_w, l->norm1_b, s->h);
    linear(s->h, T, H, l->qT, H, l->q_b, s->q);
    linear(s->h, T, H, l->kT, H, NULL, s->k); /* no key bias (reference.rs:100) */
    linear(s->h, T, H, l->vT, H, l->v_b, s->v);
    /* RoPE on patch tokens of q and k (reference.rs:108-128) */
    double *qk[2] = {s->q, s->k};
    for (int which = 0; which < 2; which++) {
      double *vals = qk[which];
      for (int token = PREFIX; token < T; token++) {
        int patch = token - PREFIX;
        for (int head = 0; head < HEADS; head++) {
          double *base = vals + (size_t)token * H + head * HD;
          memcpy(s->orig, base, HD * sizeof(double));
          for (int c = 0; c < HD; c++) {
            double rotated = c < 32 ? -s->orig[c + 32] : s->orig[c - 32];
            base[c] = s->orig[c] * s->cosv[patch * 64 + c] + rotated * s->sinv[patch * 64 + c];
          }
        }
      }
    }
    /* attention, scale 0.125 (reference.rs:129-151) */
    memset(s->ctx, 0, (size_t)T * H * sizeof(double));
    for (int head = 0; head < HEADS; head++) {
      for (int row = 0; row < T; row++) {
        const double *qr = s->q + (size_t)row * H + head * HD;
        double mx = -INFINITY;
        for (int col = 0; col < T; col++) {
          const double *kr = s->k + (size_t)col * H + head * HD;
          double dot = 0;
          for (int c = 0; c < HD; c++) dot += qr[c] * kr[c];
          s->scores[col] = dot * 0.125;
          if (s->scores[col] > mx) mx = s->scores[col];
        }
        double sum = 0;
        for (int col = 0; col < T; col++) {
          s->scores[col] = exp(s->scores[col] - mx);
          sum += s->scores[col];
        }
        double *cr = s->ctx + (size_t)row * H + head * HD;
        for (int col = 0; col < T; col++) {
          double a = s->scores[col] / sum;
          const double *vr = s->v + (size_t)col * H + head * HD;
          for (int c = 0; c < HD; c++) cr[c] += a * vr[c];
        }
      }
    }
    linear(s->ctx, T, H, l->oT, H, l->o_b, s->tmp);
    for (int i = 0; i < T * H; i++) s->x[i] += s->tmp[i] * l->ls1[i % H]; /* :159-161 */
    norm(s->x, l->norm2_w, l->norm2_b, s->h);
    linear(s->h, T, H, l->gateT, MLPH, l->gate_b, s->gate);
    linear(s->h, T, H, l->upT, MLPH, l->up_b, s->up);
    for (int i = 0; i < T * MLPH; i++) { /* SwiGLU g/(1+e^-g)*u (:177-179) */
      double g = s->gate[i];
      s->gate[i] = g / (1.0 + exp(-g)) * s->up[i];
    }
    linear(s->gate, T, MLPH, l->downT, H, l->down_b, s->tmp);
    for (int i = 0; i < T * H; i++) s->x[i] += s->tmp[i] * l->ls2[i % H]; /* :187-189 */
  }
  norm(s->x, m->norm_w, m->norm_b, out); /* :191 */
}

/* images: n x [3][224][224] float32; out: n x [201][384] float64. threads <= 0: OpenMP default.
 * Returns 0, or -1 when the model is incomplete. */
int ref_forward(const ref_model *m, const float *images, int n, double *out, int threads) {
  if (ref_model_missing(m) != 0) return -1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel
  {
    scratch s;
    size_t th = (size_t)T * H;
    s.x = malloc(th * sizeof(double));
    s.h = malloc(th * sizeof(double));
    s.q = malloc(th * sizeof(double));
    s.k = malloc(th * sizeof(double));
    s.v = malloc(th * sizeof(double));
    s.ctx = malloc(th * sizeof(double));
    s.tmp = malloc(th * sizeof(double));
    s.gate = malloc((size_t)T * MLPH * sizeof(double));
    s.up = malloc((size_t)T * MLPH * sizeof(double));
    s.patches = malloc((size_t)196 * 768 * sizeof(double));
    s.scores = malloc(T * sizeof(double));
    s.cosv = malloc(196 * 64 * sizeof(double));
    s.sinv = malloc(196 * 64 * sizeof(double));
    s.orig = malloc(HD * sizeof(double));
    ref_rope_tables(s.cosv, s.sinv);
#pragma omp for schedule(dynamic, 1)
    for (int i = 0; i < n; i++)
      forward_one(m, images + (size_t)i * 3 * 224 * 224, out + (size_t)i * T * H, &s);
    free(s.x); free(s.h); free(s.q); free(s.k); free(s.v); free(s.ctx); free(s.tmp);
    free(s.gate); free(s.up); free(s.patches); free(s.scores); free(s.cosv); free(s.sinv);
    free(s.orig);
  }
  return 0;
}

int ref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
