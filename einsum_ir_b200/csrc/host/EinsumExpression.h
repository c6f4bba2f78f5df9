// Einsum expression -> tree of EinsumNodes (interface of the reference's
// frontend::EinsumExpression, src/frontend/EinsumExpression.h:16-235) and the
// string parsers of frontend::EinsumExpressionAscii
// (src/frontend/EinsumExpressionAscii.h).
#ifndef EINSUM_IR_B200_EINSUM_EXPRESSION_H
#define EINSUM_IR_B200_EINSUM_EXPRESSION_H

#include <map>
#include <string>
#include <vector>
#include "EinsumNode.h"
#include "MemoryManager.h"
#include "constants.h"

namespace einsum_ir {
namespace frontend {

class EinsumExpression {
 public:
  //! dim id -> number of occurrences in the expression string (reference :9-23)
  static void histogram(int64_t i_num_dims, int64_t i_string_size, int64_t const *i_string_dim_ids,
                        int64_t *o_histogram);

  //! dims that survive a contraction (still used elsewhere), ascending ids (reference :25-70)
  static void substring_out(int64_t i_num_dims_left, int64_t i_num_dims_right,
                            int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                            int64_t *io_histogram, std::vector<int64_t> &o_substring_out);

  //! opt_einsum-style path (positions in the shrinking tensor list) -> unique tensor ids (reference :72-99)
  static void unique_tensor_ids(int64_t i_num_conts, int64_t const *i_path, int64_t *o_path);

  void init(int64_t i_num_dims, int64_t const *i_dim_sizes, int64_t i_num_conts,
            int64_t const *i_string_num_dims, int64_t const *i_string_dim_ids, int64_t const *i_path,
            complex_t i_ctype_ext, data_t i_dtype, void *const *i_data_ptrs);
  void init(int64_t i_num_dims, int64_t const *i_dim_sizes, int64_t i_num_conts,
            int64_t const *i_string_num_dims, int64_t const *i_string_dim_ids, int64_t const *i_path,
            data_t i_dtype, void *const *i_data_ptrs);

  err_t compile();
  err_t store_and_lock_data(int64_t i_tensor_id);
  err_t unlock_data(int64_t i_tensor_id);
  //! enqueues the whole tree on the expression's stream; returns the first error status (extension)
  int eval();
  int64_t num_ops();

  // ---- extensions of this backend
  //! data type of the input tensors (default: the expression's data type); BF16
  //! inputs give FP32 intermediates and output
  void set_input_dtype(data_t i_dtype) { m_dtype_inputs = i_dtype; }
  void set_compute_type(int32_t i_comp) { m_compute = i_comp; }
  void set_stream(void *i_stream);
  //! device pointers of the inputs followed by the output (same order as init)
  void set_data_ptrs(void *const *i_data_ptrs);
  std::vector<backend::EinsumNode> &nodes() { return m_nodes; }
  int64_t num_tensors() const { return m_num_conts + 2; }

 private:
  int64_t m_num_dims = 0;
  int64_t const *m_dim_sizes = nullptr;
  int64_t m_num_conts = 0;
  int64_t const *m_string_num_dims_ext = nullptr;
  int64_t const *m_string_dim_ids_ext = nullptr;
  int64_t const *m_path_ext = nullptr;
  complex_t m_ctype_ext = REAL_ONLY;
  data_t m_dtype = UNDEFINED_DTYPE;
  data_t m_dtype_inputs = UNDEFINED_DTYPE;
  int32_t m_compute = 0;
  void *m_stream = nullptr;
  void *const *m_data_ptrs = nullptr;
  std::vector<int64_t> m_path_int;
  std::map<int64_t, int64_t> m_map_dim_sizes;
  std::vector<int64_t> m_string_dim_ids_int;
  std::vector<int64_t> m_string_num_dims_int;
  std::vector<backend::EinsumNode> m_nodes;
  backend::MemoryManager m_memory;
  bool m_compiled = false;
};

class EinsumExpressionAscii {
 public:
  static void split_string(std::string const &i_input, std::string const &i_separation,
                           std::vector<std::string> &o_output);
  //! "iae,bf->fe" -> "[i,a,e],[b,f]->[f,e]"
  static void schar_to_standard(std::string const &i_expr_string, std::string &o_expr_string);
  //! "[x,a],[a,y]->[x,y]" -> single upper/lower-case characters per dim id
  static void standard_to_schar(std::string const &i_expr_string, std::string &o_expr_string);
  //! standard format -> tensor strings, inputs then output
  static void parse_tensors(std::string const &i_expr_string, std::vector<std::string> &o_tensors);
  static void parse_dim_sizes(std::string const &i_dim_sizes_string, std::vector<int64_t> &o_dim_sizes);
  static void parse_path(std::string const &i_expr_string, std::vector<int64_t> &o_path);
  //! dim names sorted (numbers numerically, others lexically) -> ids 0..n-1
  static void parse_dim_ids(std::string const &i_expr_string,
                            std::map<std::string, int64_t> &o_map_dim_name_to_id);
  static void parse_dtype(std::string const &i_dtype_string, data_t &o_dtype);
  static void parse_ctype(std::string const &i_ctype_string, complex_t &o_ctype);
};

}  // namespace frontend
}  // namespace einsum_ir

#endif
