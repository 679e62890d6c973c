/*
 * CPU oracle for the paged decode-attention hot path. TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference's own CPU path for one decode
 * step. It is the checker that the CUDA kernels are compared against; nothing in
 * the shipped library calls it. Only tests, the smoke check and the CPU-baseline
 * leg of bench.py load it.
 *
 * Reference algorithm followed (paths are inside tianhaoz95/unbox.ai):
 *   - unbox_platform/infer/kernels/paged_decode_attention.py:157-191
 *       paged_decode_attention_ref: for every sequence b and query head h the
 *       KV head is h // (H / KVH) (:168,175); positions pos < seq_len are gathered
 *       through block_tables[b, pos // block_size] and slot pos % block_size
 *       (:178-184); score = sum(q * k) * scale with scale = head_dim ** -0.5
 *       (:169,185); weights = softmax(scores) (:188); out = sum(w * v) (:190).
 *   - unbox_platform/infer/kvcache.py:253-262 (KVPool.write_kv) and :330-340
 *       (PagedKVCache.write_kv): block = block_table[pos // bs], slot = pos % bs,
 *       data[l, 0, block, slot] = k; data[l, 1, block, slot] = v.
 *
 * Arithmetic: inputs are widened to double and every sum is taken in double, so
 * the oracle sits closer to the exact result than the reference's fp32 torch
 * arithmetic (they agree to ~1e-7 on fp32 inputs). Softmax is the two-pass form
 * torch.softmax uses: subtract the max, exponentiate, normalise.
 *
 * Index semantics kept from the reference: a negative page id within seq_len
 * wraps like Python indexing (k_pool[-1] is the last page); an id outside
 * [-num_blocks, num_blocks) is an IndexError in the reference and an error
 * status here. seq_len == 0 makes the reference raise (torch.stack of an empty
 * list); the oracle writes zeros for that row and reports ORACLE_EMPTY_CONTEXT.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORACLE_F32 = 0, ORACLE_BF16 = 1, ORACLE_F16 = 2 };
enum {
  ORACLE_OK = 0,
  ORACLE_EMPTY_CONTEXT = 1,   /* a row had seq_len <= 0: reference raises there */
  ORACLE_BAD_PAGE = 2,        /* page id outside [-num_blocks, num_blocks)       */
  ORACLE_BAD_ARG = 3,         /* shapes / dtype not understood                    */
  ORACLE_SHORT_TABLE = 4      /* seq_len needs more pages than the table holds    */
};

static double bf16_to_double(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

/* IEEE half -> double, written from the format definition (1-5-10). */
static double f16_to_double(uint16_t h) {
  int sign = (h >> 15) & 1;
  int exp = (h >> 10) & 0x1f;
  int man = h & 0x3ff;
  double v;
  if (exp == 0) {
    v = ldexp((double)man, -24);                 /* subnormal: man * 2^-24 */
  } else if (exp == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexp((double)(man | 0x400), exp - 25);  /* (1.man) * 2^(exp-15)     */
  }
  return sign ? -v : v;
}

static double load_elem(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case ORACLE_F32: return (double)((const float*)base)[idx];
    case ORACLE_BF16: return bf16_to_double(((const uint16_t*)base)[idx]);
    default: return f16_to_double(((const uint16_t*)base)[idx]);
  }
}

static int elem_size(int dtype) { return dtype == ORACLE_F32 ? 4 : 2; }

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Threads of the parallel regions that follow (a launcher such as torchrun may
 * have set OMP_NUM_THREADS=1 for its ranks; the CPU baseline wants every core
 * it may run on). Returns the count now in effect. */
int oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
  return oracle_num_threads();
}

/*
 * Paged GQA decode attention, following paged_decode_attention.py:157-191.
 *
 * q:            (B, H, D) with element strides q_sb, q_sh (last dim contiguous)
 * k/v_cache:    (num_blocks, block_size, KVH, D) with element strides
 *               c_sblk, c_stok, c_sh (last dim contiguous)
 * block_table:  (B, max_blocks) int32, row stride bt_sb elements
 * context_lens: (B,) int32
 * out:          (B, H, D) double, contiguous
 * Work is spread over (b, kv-head) pairs with OpenMP when nthreads > 1.
 */
int oracle_paged_decode_attention(
    const void* q, int64_t q_sb, int64_t q_sh,
    const void* k_cache, const void* v_cache,
    int64_t c_sblk, int64_t c_stok, int64_t c_sh,
    const int32_t* block_table, int64_t bt_sb,
    const int32_t* context_lens,
    double* out,
    int B, int H, int KVH, int D, int block_size, int64_t num_blocks,
    int max_blocks, double scale, int dtype, int nthreads) {
  if (B < 0 || H <= 0 || KVH <= 0 || D <= 0 || block_size <= 0 || H % KVH != 0 ||
      (dtype != ORACLE_F32 && dtype != ORACLE_BF16 && dtype != ORACLE_F16))
    return ORACLE_BAD_ARG;
  const int G = H / KVH;           /* kv_repeat, paged_decode_attention.py:168 */
  int status = ORACLE_OK;
  int64_t npairs = (int64_t)B * KVH;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
  {
    int local_status = ORACLE_OK;
    int64_t cap = 0;
    double* scores = NULL;     /* (G, ctx) */
    double* qd = (double*)malloc(sizeof(double) * (size_t)G * D);
    double* acc = (double*)malloc(sizeof(double) * (size_t)G * D);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t pair = 0; pair < npairs; ++pair) {
      const int b = (int)(pair / KVH);
      const int kvh = (int)(pair % KVH);
      const int64_t ctx = context_lens[b];
      for (int g = 0; g < G; ++g) {
        const int h = kvh * G + g;   /* h // kv_repeat == kvh (:175) */
        for (int d = 0; d < D; ++d) {
          qd[(size_t)g * D + d] = load_elem(q, b * q_sb + (int64_t)h * q_sh + d, dtype);
          out[((int64_t)b * H + h) * D + d] = 0.0;
        }
      }
      if (ctx <= 0) {               /* reference: torch.stack([]) raises */
        if (local_status == ORACLE_OK) local_status = ORACLE_EMPTY_CONTEXT;
        continue;
      }
      if ((ctx + block_size - 1) / block_size > max_blocks) {
        local_status = ORACLE_SHORT_TABLE;
        continue;
      }
      if (ctx > cap) {
        free(scores);
        cap = ctx;
        scores = (double*)malloc(sizeof(double) * (size_t)G * (size_t)cap);
      }
      int bad = 0;
      /* scores: (q . k) * scale for every position (:178-185) */
      for (int64_t pos = 0; pos < ctx && !bad; ++pos) {
        int64_t page = block_table[b * bt_sb + pos / block_size];
        if (page < -num_blocks || page >= num_blocks) { bad = 1; break; }
        if (page < 0) page += num_blocks;    /* Python negative indexing */
        const int64_t base = page * c_sblk + (pos % block_size) * c_stok + (int64_t)kvh * c_sh;
        for (int g = 0; g < G; ++g) {
          double s = 0.0;
          for (int d = 0; d < D; ++d) s += qd[(size_t)g * D + d] * load_elem(k_cache, base + d, dtype);
          scores[(size_t)g * ctx + pos] = s * scale;
        }
      }
      if (bad) { local_status = ORACLE_BAD_PAGE; continue; }
      /* softmax over positions (:188), then the weighted sum of V (:190) */
      for (int g = 0; g < G; ++g) {
        double* sg = scores + (size_t)g * ctx;
        double mx = -INFINITY;
        for (int64_t pos = 0; pos < ctx; ++pos) mx = sg[pos] > mx ? sg[pos] : mx;
        double denom = 0.0;
        for (int64_t pos = 0; pos < ctx; ++pos) { sg[pos] = exp(sg[pos] - mx); denom += sg[pos]; }
        for (int64_t pos = 0; pos < ctx; ++pos) sg[pos] /= denom;
        memset(acc + (size_t)g * D, 0, sizeof(double) * D);
      }
      for (int64_t pos = 0; pos < ctx; ++pos) {
        int64_t page = block_table[b * bt_sb + pos / block_size];
        if (page < 0) page += num_blocks;
        const int64_t base = page * c_sblk + (pos % block_size) * c_stok + (int64_t)kvh * c_sh;
        for (int d = 0; d < D; ++d) {
          const double v = load_elem(v_cache, base + d, dtype);
          for (int g = 0; g < G; ++g) acc[(size_t)g * D + d] += scores[(size_t)g * ctx + pos] * v;
        }
      }
      for (int g = 0; g < G; ++g) {
        const int h = kvh * G + g;
        memcpy(out + ((int64_t)b * H + h) * D, acc + (size_t)g * D, sizeof(double) * D);
      }
    }
    free(scores);
    free(qd);
    free(acc);
#ifdef _OPENMP
#pragma omp critical
#endif
    {
      /* keep the most severe status: errors outrank the empty-context note */
      if (local_status > status) status = local_status;
    }
  }
  return status;
}

/*
 * KV append by slot mapping, following KVPool.write_kv (kvcache.py:253-262)
 * with the slot computed as PagedKVCache.write_kv does (kvcache.py:338-339):
 * slot_mapping[t] = block_table[pos // bs] * bs + pos % bs.
 * Rows are copied byte for byte. A negative slot marks a padding token and is
 * skipped. A slot at or beyond num_blocks * block_size is an error.
 */
int oracle_kv_append(
    const void* k_new, const void* v_new, int64_t n_stok, int64_t n_sh,
    void* k_cache, void* v_cache, int64_t c_sblk, int64_t c_stok, int64_t c_sh,
    const int64_t* slot_mapping, int64_t num_tokens,
    int KVH, int D, int block_size, int64_t num_blocks, int dtype) {
  if (KVH <= 0 || D <= 0 || block_size <= 0) return ORACLE_BAD_ARG;
  const int es = elem_size(dtype);
  int status = ORACLE_OK;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    if (slot >= num_blocks * block_size) { status = ORACLE_BAD_PAGE; continue; }
    const int64_t blk = slot / block_size, off = slot % block_size;
    for (int h = 0; h < KVH; ++h) {
      const int64_t src = (t * n_stok + (int64_t)h * n_sh) * es;
      const int64_t dst = (blk * c_sblk + off * c_stok + (int64_t)h * c_sh) * es;
      memcpy((char*)k_cache + dst, (const char*)k_new + src, (size_t)D * es);
      memcpy((char*)v_cache + dst, (const char*)v_new + src, (size_t)D * es);
    }
  }
  return status;
}

/*
 * Slot mapping for one decode step, the index arithmetic of
 * PagedKVCache.write_kv (kvcache.py:338-339) applied to every sequence:
 * slot[b] = block_table[b, pos // bs] * bs + pos % bs with pos = positions[b].
 * A negative position gives slot -1 (padding).
 */
int oracle_slot_mapping(const int32_t* block_table, int64_t bt_sb, const int32_t* positions,
                        int64_t* slot_mapping, int B, int max_blocks, int block_size) {
  int status = ORACLE_OK;
  for (int b = 0; b < B; ++b) {
    const int64_t pos = positions[b];
    if (pos < 0) { slot_mapping[b] = -1; continue; }
    if (pos / block_size >= max_blocks) { slot_mapping[b] = -1; status = ORACLE_SHORT_TABLE; continue; }
    const int64_t page = block_table[b * bt_sb + pos / block_size];
    slot_mapping[b] = page < 0 ? -1 : page * block_size + pos % block_size;
    if (page < 0) status = ORACLE_BAD_PAGE;
  }
  return status;
}
