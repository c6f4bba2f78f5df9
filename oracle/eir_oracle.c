/*
 * eir_oracle.c -- CPU oracle for the einsum_ir B200 backend.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates, in plain C, the semantics of
 * the reference's hot path so that the CUDA kernels can be checked against
 * it. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it; the product library never links or calls it.
 *
 * Restated reference behaviour (paths inside scalable-analyses/einsum_ir):
 *  - binary contraction loop engine: for every output point the first-touch
 *    kernel runs before the first K iteration, the main kernel accumulates
 *    left*right over all K iterations and the last-touch kernel runs after the
 *    last one (src/basic/binary/ContractionBackend.cpp:296-348, 495-515);
 *  - kernel semantics of the scalar/TPP leaves: ZERO sets 0, COPY copies the
 *    aux value, ADD adds the aux value to out, MADD accumulates l*r, RELU
 *    clamps at 0, last-touch ADD adds aux (src/basic/binary/
 *    ContractionBackendScalar.cpp:4-40, ContractionBackendTpp.cpp:15-62,130-163);
 *  - aux broadcast is expressed by stride 0 (outer size 1), as in
 *    ContractionBackendTpp.cpp:80-101 and the stride rule of
 *    src/backend/BinaryContraction.cpp:223-249;
 *  - unary permute = element copy from input strides to output strides
 *    (src/backend/Unary.cpp:3-31, src/basic/unary/UnaryBackend.cpp:106-193).
 *
 * Accumulation is in double (FP32/BF16 data) or long double (FP64 data), so
 * the oracle is at least as accurate as the reference's in-order FP32/FP64
 * accumulation. Low-precision compute types are modelled by rounding the
 * inputs first: BF16 data are exact BF16 values; TF32 compute rounds each FP32
 * input to TF32 (round to nearest, ties to even) before the product.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { O_FP32 = 0, O_FP64 = 1, O_BF16 = 2 };
enum { O_DIM_C = 0, O_DIM_M = 1, O_DIM_N = 2, O_DIM_K = 3 };
enum { O_ZERO = 0, O_RELU = 1, O_ADD = 2, O_COPY = 3, O_MADD = 4, O_UNDEF = 99 };
enum { O_COMP_DEFAULT = 0, O_COMP_FP32 = 1, O_COMP_TF32 = 2 };

#define O_MAX_DIMS 16

static double bf16_to_double(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

static float round_tf32_rne(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x; /* inf / nan */
  uint32_t lsb = (u >> 13) & 1u;
  u += 0x0fffu + lsb;
  u &= 0xffffe000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static long double load_in(const void *p, int64_t off, int dt, int comp) {
  switch (dt) {
    case O_FP64: return (long double)((const double *)p)[off];
    case O_BF16: return (long double)bf16_to_double(((const uint16_t *)p)[off]);
    default: {
      float f = ((const float *)p)[off];
      if (comp == O_COMP_TF32) f = round_tf32_rne(f);
      return (long double)f;
    }
  }
}

static long double load_out(const void *p, int64_t off, int dt) {
  return dt == O_FP64 ? (long double)((const double *)p)[off] : (long double)((const float *)p)[off];
}

static void store_out(void *p, int64_t off, int dt, long double v) {
  if (dt == O_FP64) ((double *)p)[off] = (double)v;
  else ((float *)p)[off] = (float)v;
}

/*
 * Strided binary contraction (all strides in elements).
 * Returns 0 on success, -1 on a bad argument.
 */
int eir_oracle_contract(int32_t nd, const int32_t *types, const int64_t *sizes,
                        const int64_t *sl, const int64_t *sr, const int64_t *so, const int64_t *sa,
                        int32_t dt_l, int32_t dt_r, int32_t dt_o, int32_t comp,
                        int32_t first, int32_t last,
                        const void *left, const void *right, const void *aux, void *out,
                        int32_t num_threads) {
  if (nd < 0 || nd > O_MAX_DIMS) return -1;
  int64_t osz[O_MAX_DIMS], osl[O_MAX_DIMS], osr[O_MAX_DIMS], oso[O_MAX_DIMS], osa[O_MAX_DIMS];
  int64_t ksz[O_MAX_DIMS], ksl[O_MAX_DIMS], ksr[O_MAX_DIMS];
  int no = 0, nk = 0;
  int64_t n_out = 1, n_k = 1;
  for (int i = 0; i < nd; ++i) {
    if (sizes[i] < 0) return -1;
    if (types[i] == O_DIM_K) {
      ksz[nk] = sizes[i];
      ksl[nk] = sl[i];
      ksr[nk] = sr[i];
      n_k *= sizes[i];
      ++nk;
    } else {
      osz[no] = sizes[i];
      osl[no] = types[i] == O_DIM_N ? 0 : sl[i];
      osr[no] = types[i] == O_DIM_M ? 0 : sr[i];
      oso[no] = so[i];
      osa[no] = sa ? sa[i] : 0;
      n_out *= sizes[i];
      ++no;
    }
  }
  const int use_ld = (dt_o == O_FP64);
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t g = 0; g < n_out; ++g) {
    int64_t x = g, offl = 0, offr = 0, offo = 0, offa = 0;
    for (int d = no - 1; d >= 0; --d) {
      int64_t i = x % osz[d];
      x /= osz[d];
      offl += i * osl[d];
      offr += i * osr[d];
      offo += i * oso[d];
      offa += i * osa[d];
    }
    long double v = 0.0L;
    if (first == O_COPY) v = load_out(aux, offa, dt_o);
    else if (first == O_ADD) v = load_out(out, offo, dt_o) + load_out(aux, offa, dt_o);
    else if (first != O_ZERO) v = load_out(out, offo, dt_o);
    if (use_ld) {
      long double acc = 0.0L;
      for (int64_t k = 0; k < n_k; ++k) {
        int64_t y = k, kl = 0, kr = 0;
        for (int d = nk - 1; d >= 0; --d) {
          int64_t i = y % ksz[d];
          y /= ksz[d];
          kl += i * ksl[d];
          kr += i * ksr[d];
        }
        acc += load_in(left, offl + kl, dt_l, comp) * load_in(right, offr + kr, dt_r, comp);
      }
      v += acc;
    } else {
      double acc = 0.0;
      for (int64_t k = 0; k < n_k; ++k) {
        int64_t y = k, kl = 0, kr = 0;
        for (int d = nk - 1; d >= 0; --d) {
          int64_t i = y % ksz[d];
          y /= ksz[d];
          kl += i * ksl[d];
          kr += i * ksr[d];
        }
        acc += (double)load_in(left, offl + kl, dt_l, comp) * (double)load_in(right, offr + kr, dt_r, comp);
      }
      v += (long double)acc;
    }
    if (last == O_RELU) v = v > 0.0L ? v : 0.0L;
    else if (last == O_ADD) v += load_out(aux, offa, dt_o);
    store_out(out, offo, dt_o, v);
  }
  return 0;
}

/* Permute copy: out[sum i_d*sout_d] = in[sum i_d*sin_d] (bit copy, esize bytes). */
int eir_oracle_permute(int32_t nd, const int64_t *sizes, const int64_t *sin, const int64_t *sout,
                       int32_t esize, const void *in, void *out) {
  if (nd < 0 || nd > O_MAX_DIMS || (esize != 2 && esize != 4 && esize != 8)) return -1;
  int64_t total = 1;
  for (int i = 0; i < nd; ++i) total *= sizes[i];
  for (int64_t g = 0; g < total; ++g) {
    int64_t x = g, oi = 0, oo = 0;
    for (int d = nd - 1; d >= 0; --d) {
      int64_t i = x % sizes[d];
      x /= sizes[d];
      oi += i * sin[d];
      oo += i * sout[d];
    }
    memcpy((char *)out + oo * esize, (const char *)in + oi * esize, (size_t)esize);
  }
  return 0;
}

/* TF32 rounding as the oracle models it (exposed for tests) */
void eir_oracle_round_tf32(const float *in, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = round_tf32_rne(in[i]);
}

int eir_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
