// C wrappers around the reference's own scalar contraction and permute
// backends (backend::BinaryContractionScalar over basic::ContractionBackend /
// ContractionBackendScalar, and backend::UnaryScalar), compiled from the
// reference sources where they lie (see oracle/ref.mk). TEST INFRASTRUCTURE
// ONLY: tests/ use it to pin the C oracle's numerics to the reference itself,
// and bench.py's CPU-baseline leg times it as the reference's own CPU path.
// Nothing in the product library links or loads it.
//
// The reference's loop engine reaches <libxsmm.h> only through its packing
// members (basic::UnaryBackendTpp, src/basic/binary/ContractionBackend.h:9,70-72).
// oracle/stub/libxsmm.h names the three libxsmm types that header needs; the
// three UnaryBackendTpp members below replace the libxsmm-backed ones
// (src/basic/unary/UnaryBackendTpp.cpp) and fail loudly if a plan ever asks
// for a libxsmm packing kernel.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <vector>
#include "backend/BinaryContractionScalar.h"
#include "backend/UnaryScalar.h"
#include "basic/unary/UnaryBackendTpp.h"

using einsum_ir::backend::BinaryContractionScalar;
using einsum_ir::backend::UnaryScalar;

libxsmm_datatype einsum_ir::basic::UnaryBackendTpp::dtype_to_libxsmm(data_t) {
  std::fprintf(stderr, "ref_scalar: a libxsmm packing kernel was requested (libxsmm absent)\n");
  std::abort();
}

void einsum_ir::basic::UnaryBackendTpp::kernel_main(void const *, void *) {
  std::fprintf(stderr, "ref_scalar: a libxsmm packing kernel was called (libxsmm absent)\n");
  std::abort();
}

einsum_ir::basic::err_t einsum_ir::basic::UnaryBackendTpp::compile_kernels() {
  return einsum_ir::basic::err_t::COMPILATION_FAILED;
}

namespace {

// The reference's contraction borrows every map and id array it is given
// (BinaryContraction.cpp:317-350): they live here for the plan's lifetime.
struct RefScalar {
  std::map<int64_t, int64_t> sizes, aux_outer;
  std::vector<int64_t> ids_l, ids_r, ids_o;
  BinaryContractionScalar bc;
};

einsum_ir::data_t to_dtype(int32_t d) { return d == 1 ? einsum_ir::FP64 : einsum_ir::FP32; }

einsum_ir::kernel_t to_ktype(int32_t k) {
  switch (k) {
    case 0: return einsum_ir::ZERO;
    case 1: return einsum_ir::RELU;
    case 2: return einsum_ir::ADD;
    case 3: return einsum_ir::COPY;
    case 4: return einsum_ir::MADD;
    default: return einsum_ir::UNDEFINED_KTYPE;
  }
}

}  // namespace

extern "C" {

// Creates and compiles a scalar contraction. Tensors are row-major in the
// order of their dim ids; size_ids/sizes give every dim's size; aux_outer
// (NULL: no aux) gives the aux tensor's outer size per dim of size_ids, 1 for
// a broadcast dim (the reference's stride-0 rule). dtype: 0 FP32, 1 FP64;
// ktypes use einsum_ir::kernel_t values (99 = undefined). Returns NULL when
// the reference's compile fails; *err receives its err_t.
void *ref_scalar_create(int64_t nl, int64_t nr, int64_t no, const int64_t *ids_l,
                        const int64_t *ids_r, const int64_t *ids_o, int64_t nsz,
                        const int64_t *size_ids, const int64_t *sizes, const int64_t *aux_outer,
                        int32_t dtype, int32_t first, int32_t main_k, int32_t last,
                        int64_t num_threads, int32_t *err) {
  RefScalar *p = new RefScalar();
  for (int64_t i = 0; i < nsz; ++i) {
    p->sizes[size_ids[i]] = sizes[i];
    if (aux_outer) p->aux_outer[size_ids[i]] = aux_outer[i];
  }
  p->ids_l.assign(ids_l, ids_l + nl);
  p->ids_r.assign(ids_r, ids_r + nr);
  p->ids_o.assign(ids_o, ids_o + no);
  const einsum_ir::data_t dt = to_dtype(dtype);
  p->bc.init(nl, nr, no, &p->sizes, &p->sizes, &p->sizes, aux_outer ? &p->aux_outer : nullptr,
             &p->sizes, p->ids_l.data(), p->ids_r.data(), p->ids_o.data(), dt, dt, dt, dt,
             to_ktype(first), to_ktype(main_k), to_ktype(last), num_threads);
  einsum_ir::err_t e = p->bc.compile();
  if (err) *err = (int32_t)e;
  if (e != einsum_ir::SUCCESS) {
    delete p;
    return nullptr;
  }
  return p;
}

void ref_scalar_contract(void *h, const void *l, const void *r, const void *aux, void *out) {
  RefScalar *p = static_cast<RefScalar *>(h);
  p->bc.contract(l, r, aux, out);
}

int64_t ref_scalar_num_ops(void *h) { return static_cast<RefScalar *>(h)->bc.num_ops(); }

void ref_scalar_destroy(void *h) { delete static_cast<RefScalar *>(h); }

// The reference's scalar permute (backend::UnaryScalar, COPY): out[ids_out]
// = in[ids_in], both row-major in their id order. Returns its err_t.
int32_t ref_scalar_permute(int64_t nd, const int64_t *ids_in, const int64_t *ids_out, const int64_t *size_ids,
                           const int64_t *sizes, int32_t dtype, const void *in, void *out) {
  std::map<int64_t, int64_t> sz;
  for (int64_t i = 0; i < nd; ++i) sz[size_ids[i]] = sizes[i];
  UnaryScalar u;
  const einsum_ir::data_t dt = to_dtype(dtype);
  u.init(nd, &sz, ids_in, ids_out, dt, dt, dt, einsum_ir::COPY, 1);
  einsum_ir::err_t e = u.compile();
  if (e != einsum_ir::SUCCESS) return (int32_t)e;
  u.eval(in, out);
  return 0;
}

}  // extern "C"
