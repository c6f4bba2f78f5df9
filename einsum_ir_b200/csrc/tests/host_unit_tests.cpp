// Host-side unit tests (no GPU needed): the structural known-answer cases of
// the reference's test suite, checked against this backend's host classes.
//   BinaryContraction.test.cpp:4-126   dim types, filter_dim_ids
//   EinsumExpression.test.cpp:4-60      histogram, substring_out, unique_tensor_ids
//   BinaryPrimitives.test.cpp:4-62      swap_inputs
//   EinsumExpressionAscii.test.cpp      parsers
//   MemoryManager.test.cpp:5            two-ended arena (same tree, current API names)
//   EinsumTree.test.torch.cpp:9-164     tree strings (the trees of its three cases)
#include <cstdio>
#include <iostream>
#include <map>
#include <string>
#include <vector>
#include "BinaryContraction.h"
#include "BinaryPrimitives.h"
#include "EinsumExpression.h"
#include "EinsumTree.h"
#include "MemoryManager.h"
#include "ShardedContraction.h"

using namespace einsum_ir;
using backend::BinaryContraction;
using backend::BinaryPrimitives;
using backend::MemoryManager;
using frontend::EinsumExpression;
using frontend::EinsumExpressionAscii;
using frontend::EinsumTreeAscii;

static int g_fail = 0, g_checks = 0;
#define CHECK(cond)                                                   \
  do {                                                                \
    ++g_checks;                                                       \
    if (!(cond)) {                                                    \
      ++g_fail;                                                       \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);   \
    }                                                                 \
  } while (0)

static void test_dim_types() {
  // out: i e x f g h y, left: i e a x c g y, right: a f x c h y
  int64_t out[7] = {0, 1, 2, 3, 4, 5, 6};
  int64_t left[7] = {0, 1, 7, 2, 8, 4, 6};
  int64_t right[6] = {7, 3, 2, 8, 5, 6};
  dim_t to[7], tl[7], tr[6];
  BinaryContraction::dim_types(7, 6, 7, left, right, out, UNDEFINED_DIM, M, N, C, to);
  dim_t eo[7] = {M, M, C, N, M, N, C};
  for (int i = 0; i < 7; ++i) CHECK(to[i] == eo[i]);
  BinaryContraction::dim_types(6, 7, 7, right, out, left, I, K, M, C, tl);
  dim_t el[7] = {M, M, K, C, K, M, C};
  for (int i = 0; i < 7; ++i) CHECK(tl[i] == el[i]);
  BinaryContraction::dim_types(7, 7, 6, left, out, right, J, K, N, C, tr);
  dim_t er[6] = {K, N, C, K, N, C};
  for (int i = 0; i < 6; ++i) CHECK(tr[i] == er[i]);

  int64_t ids[7] = {10, 11, 12, 13, 14, 15, 16};
  dim_t ty[7] = {M, M, C, N, M, N, C};
  int64_t f[7];
  CHECK(BinaryContraction::filter_dim_ids(7, M, ty, ids, f) == 3);
  CHECK(f[0] == 10 && f[1] == 11 && f[2] == 14);
  CHECK(BinaryContraction::filter_dim_ids(7, N, ty, ids, f) == 2);
  CHECK(f[0] == 13 && f[1] == 15);
  CHECK(BinaryContraction::filter_dim_ids(7, C, ty, ids, f) == 2);
  CHECK(f[0] == 12 && f[1] == 16);

  // dim_types_ids + strides on BASELINE config 2 (akmj,njk->anm: a is M, not C)
  int64_t a = 0, j = 1, k = 2, m = 3, n = 4;
  int64_t l2[4] = {a, k, m, j}, r2[3] = {n, j, k}, o2[3] = {a, n, m};
  std::vector<dim_t> tout;
  std::vector<int64_t> c_, m_, n_, k_, i_, j_;
  BinaryContraction::dim_types_ids(4, 3, 3, l2, r2, o2, &tout, &c_, &m_, &n_, &k_, &i_, &j_);
  CHECK(c_.empty());
  CHECK(m_.size() == 2 && m_[0] == a && m_[1] == m);
  CHECK(n_.size() == 1 && n_[0] == n);
  CHECK(k_.size() == 2 && k_[0] == k && k_[1] == j);
  std::map<int64_t, int64_t> sizes = {{a, 16}, {j, 64}, {k, 32}, {m, 512}, {n, 1}}, st;
  BinaryContraction::strides(3, o2, &sizes, &st);
  CHECK(st[m] == 1 && st[n] == 0 && st[a] == 512);  // size-1 dim gets stride 0
}

static void test_expression_helpers() {
  int64_t s[8] = {0, 2, 3, 1, 0, 4, 0, 2};
  int64_t h[5];
  EinsumExpression::histogram(5, 8, s, h);
  CHECK(h[0] == 3 && h[1] == 1 && h[2] == 2 && h[3] == 1 && h[4] == 1);

  int64_t l[4] = {1, 4, 2, 0}, r[3] = {0, 5, 2};
  int64_t hist[6] = {3, 5, 2, 7, 9, 2};
  std::vector<int64_t> sub;
  EinsumExpression::substring_out(4, 3, l, r, hist, sub);
  CHECK(sub.size() == 4);
  if (sub.size() == 4) CHECK(sub[0] == 0 && sub[1] == 1 && sub[2] == 4 && sub[3] == 5);

  int64_t path[6] = {1, 2, 2, 0, 0, 1}, up[6] = {0};
  EinsumExpression::unique_tensor_ids(3, path, up);
  CHECK(up[0] == 1 && up[1] == 2 && up[2] == 4 && up[3] == 0 && up[4] == 3 && up[5] == 5);
}

static void test_swap_inputs() {
  auto sw = [](std::vector<int64_t> l, std::vector<int64_t> r, std::vector<int64_t> o) {
    return BinaryPrimitives::swap_inputs((int64_t)l.size(), (int64_t)r.size(), (int64_t)o.size(),
                                         l.data(), r.data(), o.data());
  };
  CHECK(sw({'a', 'b'}, {'c', 'a'}, {'c', 'b'}) == false);
  CHECK(sw({'c', 'a'}, {'a', 'b'}, {'c', 'b'}) == true);
  CHECK(sw({'a', 'b', 'd'}, {'c', 'a', 'd'}, {'c', 'b', 'd'}) == false);
  CHECK(sw({'c', 'a', 'd'}, {'a', 'b', 'd'}, {'c', 'b', 'd'}) == true);
  // BASELINE config 3 / 5: the operand with the output's fastest dim becomes left
  CHECK(sw({'b', 'i'}, {'i', 'o'}, {'b', 'o'}) == true);
  CHECK(sw({'z', 'a', 'b', 'c', 'd'}, {'z', 'c', 'd', 'e', 'f'}, {'z', 'a', 'b', 'e', 'f'}) == true);
}

static void test_reorder_policy() {
  // intermediate left operand laid out [M dims in output order][K dims in the fixed right's order]
  std::map<int64_t, int64_t> sz = {{0, 4}, {1, 5}, {2, 6}, {3, 7}};
  int64_t left[3] = {2, 0, 3};   // K2, M0, K3
  int64_t right[3] = {3, 1, 2};  // K3, N1, K2 (fixed: user input)
  int64_t out[2] = {1, 0};
  CHECK(BinaryPrimitives::reorder(3, 3, 2, &sz, true, false, left, right, out) == SUCCESS);
  CHECK(left[0] == 0 && left[1] == 3 && left[2] == 2);
  CHECK(right[0] == 3 && right[1] == 1 && right[2] == 2);  // untouched
}

static void test_ascii() {
  std::string std_;
  EinsumExpressionAscii::schar_to_standard("iae,bf,dcba,cg,dh->hgfei", std_);
  CHECK(std_ == "[i,a,e],[b,f],[d,c,b,a],[c,g],[d,h]->[h,g,f,e,i]");
  std::string sc;
  EinsumExpressionAscii::standard_to_schar("[xix,a,e],[b,f],[d,c,b,a],[c,g],[d,h]->[h,g,f,e,xix]", sc);
  CHECK(sc == "IAE,BF,DCBA,CG,DH->HGFEI");
  EinsumExpressionAscii::standard_to_schar("[13,5,9],[6,10],[8,7,6,5],[7,11],[8,12]->[12,11,10,9,13]", sc);
  CHECK(sc == "IAE,BF,DCBA,CG,DH->HGFEI");
  std::vector<std::string> t;
  EinsumExpressionAscii::parse_tensors("[13,5,9],[6,10],[8,7,6,5],[7,11],[8,12]->[12,11,10,9,13]", t);
  CHECK(t.size() == 6 && t[0] == "13,5,9" && t[2] == "8,7,6,5" && t[5] == "12,11,10,9,13");
  std::map<std::string, int64_t> ids;
  EinsumExpressionAscii::parse_dim_ids("[i,aaa,e],[b,f],[d,c,b,aaa],[c,g],[d,h]->[h,g,f,e,i]", ids);
  CHECK(ids.size() == 9 && ids["aaa"] == 0 && ids["b"] == 1 && ids["e"] == 4 && ids["i"] == 8);
  EinsumExpressionAscii::parse_dim_ids("[13,5,9],[6,10],[8,7,6,5],[7,11],[8,12]->[12,11,10,9,13]", ids);
  CHECK(ids["5"] == 0 && ids["9"] == 4 && ids["10"] == 5 && ids["13"] == 8);
  std::vector<int64_t> sizes, path;
  EinsumExpressionAscii::parse_dim_sizes("32,8,4,2,16,64,8,8,8", sizes);
  CHECK(sizes.size() == 9 && sizes[0] == 32 && sizes[8] == 8);
  EinsumExpressionAscii::parse_path("(1,2),(2,3),(0,1),(0,1)", path);
  CHECK(path.size() == 8 && path[0] == 1 && path[3] == 3 && path[7] == 1);
}

static void test_memory_manager() {
  // tree of the reference's arena test: 12,20 -> 15 ; 30 -> 30 ; root 18
  MemoryManager mm;
  mm.m_layer_id++;                               // layer 1
  mm.m_layer_id++;                               // layer 2
  int64_t id1 = mm.reserve_memory(12 * 4);
  int64_t id2 = mm.reserve_memory(20 * 4);
  mm.m_layer_id--;                               // layer 1
  int64_t id3 = mm.reserve_memory(15 * 4);
  mm.remove_reservation(id1);
  mm.remove_reservation(id2);
  mm.m_layer_id++;
  int64_t id4 = mm.reserve_memory(30 * 4);
  mm.m_layer_id--;
  int64_t id5 = mm.reserve_memory(30 * 4);
  mm.remove_reservation(id4);
  mm.m_layer_id--;                               // layer 0
  int64_t id6 = mm.reserve_memory(18 * 4);
  mm.remove_reservation(id3);
  mm.remove_reservation(id5);
  CHECK(id1 >= 0 && id2 >= 0 && id3 < 0 && id4 >= 0 && id5 < 0 && id6 >= 0);
  CHECK(mm.m_req_mem >= (30 + 30 + 15) * 4);
}

static void test_tree_ascii() {
  using V = std::vector<int64_t>;
  std::string t = "[[3,0]->[0,3]],[[3,2,4],[1,4,2]->[1,2,3]]->[0,1,2]";
  int64_t n = EinsumTreeAscii::count_nodes(t);
  CHECK(n == 6);
  std::vector<V> ids(n), ch(n);
  int64_t next = 0;
  CHECK(EinsumTreeAscii::parse_tree(t, ids, ch, next) == SUCCESS && next == 6);
  std::vector<V> eids = {{3, 0}, {0, 3}, {3, 2, 4}, {1, 4, 2}, {1, 2, 3}, {0, 1, 2}};
  std::vector<V> ech = {{}, {0}, {}, {}, {2, 3}, {1, 4}};
  CHECK(ids == eids && ch == ech);
  std::map<int64_t, int64_t> sz;
  EinsumTreeAscii::parse_dim_size("2,3,4,5,6", ids, sz);
  CHECK(sz.size() == 5 && sz[0] == 2 && sz[1] == 3 && sz[2] == 4 && sz[3] == 5 && sz[4] == 6);
  CHECK(EinsumTreeAscii::count_nodes("[0,3],[1,2,3]->[0,1,2]") == 3);
  CHECK(EinsumTreeAscii::count_nodes("[0,1]->[1,0]") == 2);
  std::vector<V> i2(2), c2(2);
  next = 0;
  CHECK(EinsumTreeAscii::parse_tree("[0,1]->[1,0]", i2, c2, next) == SUCCESS && next == 2);
  CHECK(i2[1] == (V{1, 0}) && c2[1] == (V{0}));
  std::string l, r, o;
  CHECK(EinsumTreeAscii::split_outer_operation("[0,3],[1,2,3]->[0,1,2]", l, r, o) == SUCCESS);
  CHECK(l == "0,3" && r == "1,2,3" && o == "0,1,2");
  std::vector<V> bad(2), badc(2);
  next = 0;
  CHECK(EinsumTreeAscii::parse_tree("[0,1]>[1,0]", bad, badc, next) != SUCCESS);
}

// --cases: read one case per line from stdin and print this backend's answer
// (used by the test suite to compare against the reference's own functions):
//   T nl nr no <ids...>   -> dim types of left, right, out
//   S nl nr no <ids...>   -> swap_inputs (0/1)
//   U n <path...>         -> unique_tensor_ids
//   B nl nr nh <ids...> <hist...> -> substring_out
//   D <expression>        -> parse_dim_ids as name:id;...
//   E <tree> <sizes>      -> tree nodes as "ids:children;" ... "|id=size," (or -1)
static int run_cases() {
  std::string tag;
  while (std::cin >> tag) {
    if (tag == "T" || tag == "S") {
      int64_t nl, nr, no;
      std::cin >> nl >> nr >> no;
      std::vector<int64_t> l(nl), r(nr), o(no);
      for (auto &x : l) std::cin >> x;
      for (auto &x : r) std::cin >> x;
      for (auto &x : o) std::cin >> x;
      if (tag == "S") {
        std::cout << (BinaryPrimitives::swap_inputs(nl, nr, no, l.data(), r.data(), o.data()) ? 1 : 0)
                  << "\n";
      } else {
        std::vector<dim_t> tl, tr, to;
        BinaryContraction::dim_types(nl, nr, no, l.data(), r.data(), o.data(), &tl, &tr, &to);
        for (auto t : tl) std::cout << (int)t << " ";
        for (auto t : tr) std::cout << (int)t << " ";
        for (auto t : to) std::cout << (int)t << " ";
        std::cout << "\n";
      }
    } else if (tag == "U") {
      int64_t n;
      std::cin >> n;
      std::vector<int64_t> p(2 * n), u(2 * n);
      for (auto &x : p) std::cin >> x;
      EinsumExpression::unique_tensor_ids(n, p.data(), u.data());
      for (auto x : u) std::cout << x << " ";
      std::cout << "\n";
    } else if (tag == "B") {
      int64_t nl, nr, nh;
      std::cin >> nl >> nr >> nh;
      std::vector<int64_t> l(nl), r(nr), h(nh), s;
      for (auto &x : l) std::cin >> x;
      for (auto &x : r) std::cin >> x;
      for (auto &x : h) std::cin >> x;
      EinsumExpression::substring_out(nl, nr, l.data(), r.data(), h.data(), s);
      for (auto x : s) std::cout << x << " ";
      std::cout << "\n";
    } else if (tag == "D") {
      std::string e;
      std::cin >> e;
      std::map<std::string, int64_t> ids;
      EinsumExpressionAscii::parse_dim_ids(e, ids);
      for (auto const &kv : ids) std::cout << kv.first << ":" << kv.second << ";";
      std::cout << "\n";
    } else if (tag == "E") {
      std::string t, sizes;
      std::cin >> t >> sizes;
      int64_t n = EinsumTreeAscii::count_nodes(t), next = 0;
      std::vector<std::vector<int64_t>> ids(n), ch(n);
      if (EinsumTreeAscii::parse_tree(t, ids, ch, next) != SUCCESS || next != n) {
        std::cout << "-1\n";
      } else {
        std::map<int64_t, int64_t> sz;
        EinsumTreeAscii::parse_dim_size(sizes, ids, sz);
        for (int64_t i = 0; i < n; ++i) {
          for (auto x : ids[i]) std::cout << x << ",";
          std::cout << ":";
          for (auto x : ch[i]) std::cout << x << ",";
          std::cout << ";";
        }
        std::cout << "|";
        for (auto const &kv : sz) std::cout << kv.first << "=" << kv.second << ",";
        std::cout << "\n";
      }
    }
    std::cout.flush();
  }
  return 0;
}

// ShardedContraction planning (no GPU needed): BASELINE config 5 over 4
// ranks, the block of rank 2, the whole job's flops, and the layouts it
// refuses (sharded dim not outermost, not divisible by the ranks)
static void test_sharded_contraction() {
  using einsum_ir::backend::ShardedContraction;
  std::map<int64_t, int64_t> sizes;
  for (int64_t d = 0; d < 6; ++d) sizes[d] = 48;
  sizes[6] = 64;
  int64_t l[5] = {6, 0, 1, 2, 3}, r[5] = {6, 2, 3, 4, 5}, o[5] = {6, 0, 1, 4, 5};
  ShardedContraction sc;
  sc.init(5, 5, 5, &sizes, l, r, o, FP64, 6, 2, 4);
  CHECK(sc.compile() == SUCCESS);
  CHECK(sc.block_size() == 16 && sc.block_begin() == 32);
  CHECK(sc.slab_bytes() == 48 * 48 * 48 * 48 * 8);
  CHECK(sc.num_ops() == 2 * 64 * 2304LL * 2304LL * 2304LL - 64 * 2304LL * 2304LL);  // ZERO first touch
  CHECK(sc.contract(nullptr, nullptr, nullptr) == EIR_INVALID_ARGUMENT);  // bind_output first
  ShardedContraction bad_dim;
  int64_t o2[5] = {0, 6, 1, 4, 5};
  bad_dim.init(5, 5, 5, &sizes, l, r, o2, FP64, 6, 0, 4);
  CHECK(bad_dim.compile() != SUCCESS);
  ShardedContraction bad_split;
  bad_split.init(5, 5, 5, &sizes, l, r, o, FP64, 6, 0, 3);
  CHECK(bad_split.compile() != SUCCESS);
  // a one-rank output group maps nothing and has no peers
  double buf[4] = {0, 0, 0, 0};
  eir_output_group *g = nullptr;
  CHECK(eir_output_group_create(0, 1, buf, nullptr, nullptr, &g) == EIR_SUCCESS && g != nullptr);
  CHECK(eir_output_group_peers(g, 16, nullptr) == EIR_SUCCESS);
  CHECK(eir_output_group_destroy(g) == EIR_SUCCESS);
  CHECK(eir_output_group_create(1, 1, buf, nullptr, nullptr, &g) == EIR_INVALID_ARGUMENT);
}

int main(int argc, char **argv) {
  if (argc > 1 && std::string(argv[1]) == "--cases") return run_cases();
  test_sharded_contraction();
  test_dim_types();
  test_expression_helpers();
  test_swap_inputs();
  test_reorder_policy();
  test_ascii();
  test_tree_ascii();
  test_memory_manager();
  std::printf("%d checks, %d failed\n", g_checks, g_fail);
  return g_fail == 0 ? 0 : 1;
}
