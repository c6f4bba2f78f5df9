// Strided binary contraction interface (host side of the drop-in boundary).
//
// Same public interface as the reference's einsum_ir::backend::BinaryContraction
// (src/backend/BinaryContraction.h:16-392): the public members drivers read
// (m_num_dims_{c,m,n,k}, m_sizes_{c,m,n,k}, ...), the static helpers
// dim_types / filter_dim_ids / dim_types_ids / strides, the two init
// overloads, compile_base, the virtual compile / contract and num_ops.
// All pointers handed to init are borrowed and must outlive compile/contract.
#ifndef EINSUM_IR_B200_BINARY_CONTRACTION_H
#define EINSUM_IR_B200_BINARY_CONTRACTION_H

#include <cstdint>
#include <map>
#include <vector>
#include "MemoryManager.h"
#include "constants.h"

namespace einsum_ir {
namespace backend {

class BinaryContraction {
 public:
  int64_t m_num_dims_left = 0;
  int64_t m_num_dims_right = 0;
  int64_t m_num_dims_out = 0;

  std::map<int64_t, int64_t> const *m_dim_sizes_inner = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_outer_left = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_outer_right = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_outer_out_aux = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_outer_out = nullptr;

  std::map<int64_t, dim_t> m_dim_types;

  int64_t const *m_dim_ids_left = nullptr;
  int64_t const *m_dim_ids_right = nullptr;
  int64_t const *m_dim_ids_out = nullptr;

  int64_t const *m_dim_ids_permute_left = nullptr;
  int64_t const *m_dim_ids_permute_right = nullptr;

  std::vector<int64_t> const *m_loop_ids_ext = nullptr;
  std::vector<int64_t> m_loop_ids_int;

  std::vector<dim_t> m_dim_types_out;

  int64_t m_num_dims_c = 0, m_num_dims_m = 0, m_num_dims_n = 0, m_num_dims_k = 0;
  int64_t m_num_dims_i = 0, m_num_dims_j = 0;

  std::vector<int64_t> m_dim_ids_c, m_dim_ids_m, m_dim_ids_n, m_dim_ids_k, m_dim_ids_i, m_dim_ids_j;
  std::vector<int64_t> m_sizes_c, m_sizes_m, m_sizes_n, m_sizes_k, m_sizes_i, m_sizes_j;

  data_t m_dtype_left = UNDEFINED_DTYPE;
  data_t m_dtype_right = UNDEFINED_DTYPE;
  data_t m_dtype_comp = UNDEFINED_DTYPE;
  data_t m_dtype_out = UNDEFINED_DTYPE;

  kernel_t m_ktype_first_touch = UNDEFINED_KTYPE;
  kernel_t m_ktype_main = UNDEFINED_KTYPE;
  kernel_t m_ktype_last_touch = UNDEFINED_KTYPE;

  bool m_compiled = false;
  MemoryManager *m_memory = nullptr;
  int64_t m_num_threads = 1;

  // Type of every dim of tensor t2 relative to t0 and t1: exclusive to t2,
  // shared with t0 only, with t1 only, or with both (reference :7-61).
  static void dim_types(int64_t i_num_dims_t0, int64_t i_num_dims_t1, int64_t i_num_dims_t2,
                        int64_t const *i_dim_ids_t0, int64_t const *i_dim_ids_t1,
                        int64_t const *i_dim_ids_t2, dim_t i_dim_type_t2, dim_t i_dim_type_t2_t0,
                        dim_t i_dim_type_t2_t1, dim_t i_dim_type_t2_t0_t1, dim_t *o_dim_types_t2);

  // Dim types of left (I/K/M/C), right (J/K/N/C) and out (M/N/C) (reference :63-111).
  static void dim_types(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                        int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                        int64_t const *i_dim_ids_out, std::vector<dim_t> *o_dim_types_left,
                        std::vector<dim_t> *o_dim_types_right, std::vector<dim_t> *o_dim_types_out);

  static int64_t filter_dim_ids(int64_t i_num_dims_tensor, dim_t i_dim_type_filter,
                                dim_t const *i_dim_types_tensor, int64_t const *i_dim_ids_tensor,
                                int64_t *o_dim_ids_filtered);

  // C/M/N ids in output order, K/I ids in left order, J ids in right order (reference :131-221).
  static void dim_types_ids(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                            int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                            int64_t const *i_dim_ids_out, std::vector<dim_t> *o_dim_types_out,
                            std::vector<int64_t> *o_dim_ids_c, std::vector<int64_t> *o_dim_ids_m,
                            std::vector<int64_t> *o_dim_ids_n, std::vector<int64_t> *o_dim_ids_k,
                            std::vector<int64_t> *o_dim_ids_i, std::vector<int64_t> *o_dim_ids_j);

  // Row-major strides from the (outer) sizes; dims of size < 2 get stride 0 (reference :223-249).
  static void strides(int64_t i_num_dims, int64_t const *i_dim_ids,
                      std::map<int64_t, int64_t> const *i_dim_sizes,
                      std::map<int64_t, int64_t> *o_strides);

  virtual ~BinaryContraction() {}

  void init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
            std::map<int64_t, int64_t> const *i_dim_sizes_inner,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_left,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_right,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_out_aux,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_out, int64_t const *i_dim_ids_left,
            int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out, data_t i_dtype_left,
            data_t i_dtype_right, data_t i_dtype_comp, data_t i_dtype_out,
            kernel_t i_ktype_first_touch, kernel_t i_ktype_main, kernel_t i_ktype_last_touch,
            int64_t i_num_threads);

  void init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
            std::map<int64_t, int64_t> const *i_dim_sizes_inner,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_left,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_right,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_out_aux,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer_out,
            std::vector<int64_t> const *i_loop_ids_ext, int64_t const *i_dim_ids_left,
            int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out,
            int64_t const *i_dim_ids_permute_left, int64_t const *i_dim_ids_permute_right,
            MemoryManager *i_memory, data_t i_dtype_left, data_t i_dtype_right, data_t i_dtype_comp,
            data_t i_dtype_out, kernel_t i_ktype_first_touch, kernel_t i_ktype_main,
            kernel_t i_ktype_last_touch, int64_t i_num_threads);

  err_t compile_base();

  virtual err_t compile() = 0;

  virtual void contract(void const *i_tensor_left, void const *i_tensor_right,
                        void *io_tensor_out) = 0;

  virtual void contract(void const *i_tensor_left, void const *i_tensor_right,
                        void const *i_tensor_out_aux, void *io_tensor_out) = 0;

  // 2*|C||M||N||K|, minus |C||M||N| for a ZERO first touch (reference :434-465)
  int64_t num_ops();
};

}  // namespace backend
}  // namespace einsum_ir

#endif
