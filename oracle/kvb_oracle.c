/* TEST INFRASTRUCTURE - the FP64 CPU oracle of kvbridge decode attention.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
 * this file, and only as the checker. The product path (libkvbridge_b200.so)
 * never calls it.
 *
 * Restates kvbridge_example::reference() of the reference repository
 * (examples/attention_reference.h:53-89) in C with the same double-precision
 * operation order, so that on identical inputs it reproduces the reference's
 * own oracle bit for bit (checked against the reference's oracle compiled
 * from its sources into oracle/_ref, see oracle/Makefile):
 *   logit_t = (sum_d (double)q*(double)k*(double)ks) * (double)scale  if kpos_t <= qpos_r
 *           = -inf                                                    otherwise
 *   out[d]  = (sum_t exp(logit_t - max) * (double)v * (double)vs) / sum_t exp(logit_t - max)
 * Extensions beyond the reference oracle (marked below): it also returns the
 * max logit m and denominator l of each row-head, accepts fp32 K/V
 * (int8 == 0, no scales), and splits the row-heads over pthreads. */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct kvbo_shape {
  uint32_t rows, q_heads, kv_heads, dim, page_tokens, pages, tokens, begin, end;
  float scale;
  int32_t int8;
} kvbo_shape;

typedef struct kvbo_inputs {
  const float* q;
  const int64_t* q_positions;
  const int64_t* k_positions;
  const uint32_t* page_table;
  const void* k;
  const void* v;
  const float* k_scales;
  const float* v_scales;
} kvbo_inputs;

typedef struct kvbo_outputs {
  double* normalized; /* [rows*q_heads*dim], zero for invisible row-heads */
  double* m;          /* [rows*q_heads] max logit, -inf if invisible (extension) */
  double* l;          /* [rows*q_heads] softmax denominator, 0 if invisible (extension) */
  uint8_t* visible;   /* [rows*q_heads] */
} kvbo_outputs;

typedef struct task {
  const kvbo_shape* s;
  const kvbo_inputs* in;
  const kvbo_outputs* out;
  uint32_t rh_begin, rh_end;
  int status;
} task;

static double k_value(const kvbo_shape* s, const kvbo_inputs* in, size_t i) {
  return s->int8 ? (double)((const int8_t*)in->k)[i] : (double)((const float*)in->k)[i];
}
static double v_value(const kvbo_shape* s, const kvbo_inputs* in, size_t i) {
  return s->int8 ? (double)((const int8_t*)in->v)[i] : (double)((const float*)in->v)[i];
}

/* One (row, head): reference examples/attention_reference.h:60-88. */
static void row_head(const kvbo_shape* s, const kvbo_inputs* in, const kvbo_outputs* out,
                     uint32_t rh, double* logits) {
  const uint32_t group = s->q_heads / s->kv_heads;
  const uint32_t r = rh / s->q_heads, h = rh % s->q_heads;
  const uint32_t kv = h / group;
  const uint32_t P = s->page_tokens, D = s->dim;
  double maximum = -INFINITY;
  int visible = 0;
  for (uint32_t t = s->begin; t < s->end; ++t) {
    double dot = -INFINITY;
    if (in->k_positions[t] <= in->q_positions[r]) {
      const size_t si = ((size_t)in->page_table[t / P] * s->kv_heads + kv) * P + t % P;
      const double ks = s->int8 ? (double)in->k_scales[si] : 1.0;
      dot = 0;
      for (uint32_t d = 0; d < D; ++d)
        dot += (double)in->q[(size_t)rh * D + d] * k_value(s, in, si * D + d) * ks;
      dot *= (double)s->scale;
      visible = 1;
    }
    logits[t - s->begin] = dot;
    if (maximum < dot) maximum = dot; /* std::max(maximum, dot) */
  }
  double* o = out->normalized + (size_t)rh * D;
  for (uint32_t d = 0; d < D; ++d) o[d] = 0;
  out->visible[rh] = (uint8_t)visible;
  if (out->m) out->m[rh] = visible ? maximum : -INFINITY;
  if (out->l) out->l[rh] = 0;
  if (!visible) return;
  double denominator = 0;
  for (uint32_t t = s->begin; t < s->end; ++t) {
    const double weight = exp(logits[t - s->begin] - maximum);
    denominator += weight;
    const uint32_t p = in->page_table[t / P], slot = t % P;
    const size_t si = ((size_t)p * s->kv_heads + kv) * P + slot;
    const double vs = s->int8 ? (double)in->v_scales[si] : 1.0;
    const size_t vbase = ((size_t)p * s->kv_heads + kv) * D * P + slot;
    for (uint32_t d = 0; d < D; ++d) o[d] += weight * v_value(s, in, vbase + (size_t)d * P) * vs;
  }
  for (uint32_t d = 0; d < D; ++d) o[d] /= denominator;
  if (out->l) out->l[rh] = denominator;
}

static void* run_task(void* arg) {
  task* t = (task*)arg;
  const size_t span = t->s->end > t->s->begin ? t->s->end - t->s->begin : 1;
  double* logits = (double*)malloc(span * sizeof(double));
  if (!logits) {
    t->status = 2;
    return NULL;
  }
  for (uint32_t rh = t->rh_begin; rh < t->rh_end; ++rh) row_head(t->s, t->in, t->out, rh, logits);
  free(logits);
  t->status = 0;
  return NULL;
}

/* Returns 0 on success, 1 on invalid arguments, 2 on allocation/thread failure.
 * Metadata validity (kvbridge::attention_shape_error) is the caller's job, as
 * in the reference, which validates before calling its oracle. */
int kvbo_reference(const kvbo_shape* s, const kvbo_inputs* in, const kvbo_outputs* out,
                   int threads) {
  if (!s || !in || !out || !out->normalized || !out->visible) return 1;
  if (!s->kv_heads || s->q_heads % s->kv_heads || !s->page_tokens) return 1;
  const uint32_t rhs = s->rows * s->q_heads;
  if (threads < 1) threads = 1;
  if ((uint32_t)threads > rhs) threads = rhs ? (int)rhs : 1;
  task* tasks = (task*)calloc((size_t)threads, sizeof(task));
  pthread_t* ids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!tasks || !ids) {
    free(tasks);
    free(ids);
    return 2;
  }
  int status = 0;
  for (int i = 0; i < threads; ++i) {
    tasks[i].s = s;
    tasks[i].in = in;
    tasks[i].out = out;
    tasks[i].rh_begin = (uint32_t)((uint64_t)rhs * i / threads);
    tasks[i].rh_end = (uint32_t)((uint64_t)rhs * (i + 1) / threads);
    tasks[i].status = 2;
  }
  int started = 0;
  for (int i = 1; i < threads; ++i) {
    if (pthread_create(&ids[i], NULL, run_task, &tasks[i]) != 0) {
      status = 2;
      break;
    }
    started = i;
  }
  run_task(&tasks[0]);
  for (int i = 1; i <= started; ++i) pthread_join(ids[i], NULL);
  for (int i = 0; i < threads && status == 0; ++i) status = tasks[i].status;
  free(tasks);
  free(ids);
  return status;
}

/* Log-sum-exp merge of `parts` partials (m, l, n[dim]) per row-head in FP64,
 * the algebra of reference src/attention_shared.cu:295-335 (partials with
 * l <= 0 are skipped). Layout: m/l [parts][rh], n [parts][rh][dim]. */
void kvbo_merge(uint32_t parts, uint32_t row_heads, uint32_t dim, const double* m,
                const double* l, const double* n, double* m_out, double* l_out,
                double* n_out) {
  for (uint32_t rh = 0; rh < row_heads; ++rh) {
    double M = -INFINITY;
    for (uint32_t p = 0; p < parts; ++p) {
      const size_t i = (size_t)p * row_heads + rh;
      if (l[i] > 0 && m[i] > M) M = m[i];
    }
    double L = 0;
    double* o = n_out + (size_t)rh * dim;
    for (uint32_t d = 0; d < dim; ++d) o[d] = 0;
    if (M != -INFINITY) {
      for (uint32_t p = 0; p < parts; ++p) {
        const size_t i = (size_t)p * row_heads + rh;
        if (!(l[i] > 0)) continue;
        const double e = exp(m[i] - M);
        L += e * l[i];
        for (uint32_t d = 0; d < dim; ++d) o[d] += e * n[i * dim + d];
      }
    }
    m_out[rh] = L > 0 ? M : -INFINITY;
    l_out[rh] = L;
  }
}

/* Paged KV append (no counterpart in the reference, which ships no
 * quantiser; the rule is the benchmark configurations' symmetric
 * per-(token, kv-head) absmax quantisation): for each of `tokens` rows and
 * kv head h, K row x = k_new[(t*kv_heads + h)*dim ..], likewise V,
 *   scale = max|x| / 127 (float), div = scale > 0 ? scale : 1,
 *   code  = clamp(rint(x / div), -127, 127)   (float division, ties to even)
 * written to physical slot slots[t] = page*page_tokens + s of the pool in the
 * reference layout (attention_common.h:11-46): K codes at
 * ((page*kv_heads + h)*P + s)*dim + d, V codes at ((page*kv_heads + h)*dim +
 * d)*P + s, scales at (page*kv_heads + h)*P + s. Negative slots are skipped;
 * slots >= pages*P are skipped and counted (the return value). */
int kvbo_append_kv(uint32_t tokens, uint32_t kv_heads, uint32_t dim, uint32_t page_tokens,
                   uint32_t pages, const float* k_new, const float* v_new, const int64_t* slots,
                   int8_t* k, int8_t* v, float* k_scales, float* v_scales) {
  int bad = 0;
  const uint64_t P = page_tokens, total = (uint64_t)pages * page_tokens;
  for (uint32_t t = 0; t < tokens; ++t) {
    if (slots[t] < 0) continue;
    if ((uint64_t)slots[t] >= total) {
      ++bad;
      continue;
    }
    const uint64_t page = (uint64_t)slots[t] / P, s = (uint64_t)slots[t] % P;
    for (uint32_t h = 0; h < kv_heads; ++h) {
      const uint64_t unit = page * kv_heads + h;
      for (int kind = 0; kind < 2; ++kind) {
        const float* x = (kind == 0 ? k_new : v_new) + ((uint64_t)t * kv_heads + h) * dim;
        float amax = 0.0f;
        for (uint32_t d = 0; d < dim; ++d) {
          const float a = fabsf(x[d]);
          if (a > amax) amax = a;
        }
        const float scale = amax / 127.0f;
        const float div = scale > 0.0f ? scale : 1.0f;
        for (uint32_t d = 0; d < dim; ++d) {
          float c = rintf(x[d] / div);
          if (c > 127.0f) c = 127.0f;
          if (c < -127.0f) c = -127.0f;
          if (kind == 0)
            k[(unit * P + s) * dim + d] = (int8_t)(int)c;
          else
            v[(unit * dim + d) * P + s] = (int8_t)(int)c;
        }
        (kind == 0 ? k_scales : v_scales)[unit * P + s] = scale;
      }
    }
  }
  return bad;
}
