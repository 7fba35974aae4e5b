// The reference's own unit tests for the hot path (src/linalg/tensor/ops.rs,
// src/linalg/tensor/base.rs, src/activation), restated against the C++ mirror
// of Tensor<T> (include/trs_tensor.hpp) running on the GPU through the C ABI.
// Each test keeps the name of the reference test it restates.
#include <cmath>
#include <cstdio>
#include <functional>
#include <string>
#include <vector>

#include "trs_tensor.hpp"

using trs::Tensor;
using V = std::vector<int64_t>;

static int g_failures = 0;
#define CHECK(cond)                                                              \
  do {                                                                           \
    if (!(cond)) {                                                               \
      std::fprintf(stderr, "  %s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
      throw std::runtime_error("check failed");                                   \
    }                                                                            \
  } while (0)

template <class T>
static Tensor<T> t1(std::vector<T> d) { V s{(int64_t)d.size()}; return Tensor<T>::new_(d, s); }
template <class T>
static Tensor<T> t2(std::vector<T> d, int64_t r, int64_t c) { return Tensor<T>::new_(d, V{r, c}); }

// ---- ops.rs:511-612 ----
static void add_test() {
  auto a = t1<int32_t>({1, 2, 3});
  auto b = t1<int32_t>({3, 4, 5});
  auto c = a + b;
  CHECK(c.get_shape() == V{3});
  CHECK((c.get_data() == std::vector<int32_t>{4, 6, 8}));
}

static void scalar_broadcast_add() {
  auto a = t1<int32_t>({1, 2, 3, 4});
  auto b = t1<int32_t>({10});
  auto c = a + b;
  CHECK(c.get_shape() == V{4});
  CHECK((c.get_data() == std::vector<int32_t>{11, 12, 13, 14}));
}

static void vector_matrix_broadcast_add() {
  auto a = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto b = t2<int32_t>({10, 20, 30}, 1, 3);
  auto c = a + b;
  CHECK((c.get_shape() == V{2, 3}));
  CHECK((c.get_data() == std::vector<int32_t>{11, 22, 33, 14, 25, 36}));
}

static void broadcast_disables_inplace() {
  auto a = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto b = t1<int32_t>({10, 20, 30});
  auto c = a + b;
  CHECK((a.get_data() == std::vector<int32_t>{1, 2, 3, 4, 5, 6}));
  CHECK((c.get_data() == std::vector<int32_t>{11, 22, 33, 14, 25, 36}));
}

static void add_assign_no_broadcast() {
  auto a = t1<int32_t>({1, 2, 3});
  auto b = t1<int32_t>({10, 20, 30});
  a += b;
  CHECK(a.get_shape() == V{3});
  CHECK((a.get_data() == std::vector<int32_t>{11, 22, 33}));
}

static void view_then_materialize() {
  auto a = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto b = *a.slice({0, 1}, {2, 2});
  CHECK(!b.is_contiguous());
  auto c = b.clone();
  CHECK(c.is_contiguous());
  CHECK((c.get_shape() == V{2, 2}));
  CHECK((c.get_data() == std::vector<int32_t>{2, 3, 5, 6}));
}

// ---- base.rs:2133-2301 ----
static void transpose_view() {
  auto a = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto t = a.transpose();
  CHECK((t.get_shape() == V{3, 2}));
  CHECK(!t.is_contiguous());
  CHECK((t.get_data() == std::vector<int32_t>{1, 4, 2, 5, 3, 6}));
}

static void sum_axis() {
  auto a = Tensor<float>::new_({0, 1, 2, 3}, V{2, 2});
  auto b = *a.slice({1, 0}, {1, 2});
  auto what = b.sum_axis_keepdim(0);
  CHECK((what.get_shape() == V{1, 2}));
  CHECK((what.get_data() == std::vector<float>{2.0f, 3.0f}));
  auto x = t2<double>({1, 2, 3, 4, 5, 6}, 2, 3);
  CHECK((x.sum_axis(0).get_data() == std::vector<double>{5, 7, 9}));
  CHECK((x.sum_axis(1).get_data() == std::vector<double>{6, 15}));
}

static void strided_1d_view_is_not_contiguous() {
  auto a = Tensor<int32_t>::new_({1, 2, 3, 4, 5, 6}, V{6});
  auto strided = *a.step_slice({0}, {3}, {2});
  CHECK((strided.get_data() == std::vector<int32_t>{1, 3, 5}));
  CHECK(!strided.is_contiguous());
  CHECK(Tensor<int32_t>::scalar(1).is_contiguous());
  CHECK(a.reshape({1, 6, 1}).is_contiguous());
}

static void reduce_broadcast_grad_keeps_target_rank() {
  auto grad = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto g = *grad.reduce_broadcast_grad({3});
  CHECK(g.get_shape() == V{3});
  CHECK((g.get_data() == std::vector<int32_t>{5, 7, 9}));
  g = *grad.reduce_broadcast_grad({1, 3});
  CHECK((g.get_shape() == V{1, 3}));
  CHECK((g.get_data() == std::vector<int32_t>{5, 7, 9}));
  g = *grad.reduce_broadcast_grad({2, 1});
  CHECK((g.get_shape() == V{2, 1}));
  CHECK((g.get_data() == std::vector<int32_t>{6, 15}));
  g = *grad.reduce_broadcast_grad({1, 1});
  CHECK((g.get_shape() == V{1, 1}));
  CHECK((g.get_data() == std::vector<int32_t>{21}));
  auto batched = Tensor<int32_t>::new_({1, 2, 3, 4, 5, 6, 7, 8}, V{2, 2, 2});
  g = *batched.reduce_broadcast_grad({2, 2});
  CHECK((g.get_shape() == V{2, 2}));
  CHECK((g.get_data() == std::vector<int32_t>{6, 8, 10, 12}));
  CHECK(!grad.reduce_broadcast_grad({2, 2}).has_value());
}

// ---- doctests of base.rs ----
static void doctests() {
  auto a = Tensor<int32_t>::new_({1, 2, 3, 4}, V{2, 2});
  CHECK(a.sum().item() == 10);                                               // base.rs:1022
  auto b = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  CHECK((b.sum_axis(0).get_data() == std::vector<int32_t>{5, 7, 9}));       // base.rs:1039
  CHECK((b.sum_axis(1).get_data() == std::vector<int32_t>{6, 15}));         // base.rs:1040
  auto m = t2<int32_t>({1, 5, 3, 4, 2, 6}, 2, 3);
  CHECK((m.max_axis(1).get_data() == std::vector<int32_t>{5, 6}));          // base.rs:1239
  CHECK((m.max_axis(0).get_data() == std::vector<int32_t>{4, 5, 6}));       // base.rs:1240
  CHECK((m.argmax_axis(1) == std::vector<int64_t>{1, 2}));                   // base.rs:1446
  auto r = Tensor<int32_t>::new_({1, 2, 3, 4, 5, 6}, V{6});
  CHECK((r.step_slice({5}, {6}, {-1})->get_data() == std::vector<int32_t>{6, 5, 4, 3, 2, 1}));  // base.rs:358
  CHECK((b.permute({1, 0})->get_data() == std::vector<int32_t>{1, 4, 2, 5, 3, 6}));              // base.rs:497
  CHECK((b.slice({1, 0}, {1, 3})->get_data() == std::vector<int32_t>{4, 5, 6}));                // base.rs:311
  CHECK(b.get({1, 0}).value() == 4 && !b.get({2, 0}).has_value() && !b.get({0}).has_value());
}

// ---- activation/mod.rs:229-289, activation/softmax.rs:88-153 ----
static void tanh_saturates_instead_of_overflowing() {
  auto x = Tensor<float>::new_({0, 20, 50, 90, 300, -300}, V{1, 6});
  auto y = x.tanh();
  CHECK((y.get_data() == std::vector<float>{0, 1, 1, 1, 1, -1}));
}

static void sigmoid_stays_finite_on_both_sides() {
  auto x = Tensor<float>::new_({0, 100, -100, 400, -400}, V{1, 5});
  auto v = x.sigmoid().get_data();
  CHECK(v[0] == 0.5f && v[1] == 1.0f && v[2] < 1e-40f && v[2] >= 0.0f && v[3] == 1.0f && v[4] == 0.0f);
}

static void test_activations_forward() {
  auto x = Tensor<float>::new_({-1, 0, 1}, V{1, 3});
  CHECK((x.relu().get_data() == std::vector<float>{0, 0, 1}));
  CHECK((x.leaky_relu(0.1f).get_data() == std::vector<float>{-0.1f, 0, 1}));
  CHECK(std::fabs(x.sigmoid().get_data()[1] - 0.5f) < 1e-5f);
  CHECK(std::fabs(x.tanh().get_data()[1] - 0.0f) < 1e-5f);
}

static void test_softmax_logic() {
  auto x = Tensor<float>::new_({1, 2, 3}, V{1, 3});
  auto d = x.softmax().get_data();
  CHECK(std::fabs(d[0] + d[1] + d[2] - 1.0f) < 1e-5f);
  CHECK(d[2] > d[1] && d[1] > d[0]);
}

static void test_selu_scaling() {
  auto x = Tensor<float>::new_({1}, V{1, 1});
  CHECK(std::fabs(x.selu(1.67326f, 1.0507f).get_data()[0] - 1.0507f) < 1e-5f);
}

// ---- panics and None, as the reference reports them ----
static void errors_match_the_reference() {
  auto a = t2<int32_t>({1, 2, 3, 4, 5, 6}, 2, 3);
  auto b = t1<int32_t>({1, 2});
  try {
    (void)(a + b);
    CHECK(false);
  } catch (const trs::Panic& p) {
    CHECK(std::string(p.what()) == "!!!Add: incompatible shapes!!!");
  }
  try {
    (void)a.sum_axis(2);
    CHECK(false);
  } catch (const trs::Panic& p) {
    CHECK(std::string(p.what()) == "!!!Axis index out of range!!!");
  }
  auto e = Tensor<float>::new_({}, V{3, 0});
  try {
    (void)e.max_axis(1);
    CHECK(false);
  } catch (const trs::Panic& p) {
    CHECK(std::string(p.what()) == "!!!Cannot reduce an empty axis!!!");
  }
  CHECK(!a.permute({0, 0}).has_value());
  CHECK(!a.slice({0, 2}, {2, 2}).has_value());
}

int main() {
  const std::vector<std::pair<const char*, std::function<void()>>> tests = {
      {"add_test", add_test},
      {"scalar_broadcast_add", scalar_broadcast_add},
      {"vector_matrix_broadcast_add", vector_matrix_broadcast_add},
      {"broadcast_disables_inplace", broadcast_disables_inplace},
      {"add_assign_no_broadcast", add_assign_no_broadcast},
      {"view_then_materialize", view_then_materialize},
      {"transpose_view", transpose_view},
      {"sum_axis", sum_axis},
      {"strided_1d_view_is_not_contiguous", strided_1d_view_is_not_contiguous},
      {"reduce_broadcast_grad_keeps_target_rank", reduce_broadcast_grad_keeps_target_rank},
      {"doctests", doctests},
      {"tanh_saturates_instead_of_overflowing", tanh_saturates_instead_of_overflowing},
      {"sigmoid_stays_finite_on_both_sides", sigmoid_stays_finite_on_both_sides},
      {"test_activations_forward", test_activations_forward},
      {"test_softmax_logic", test_softmax_logic},
      {"test_selu_scaling", test_selu_scaling},
      {"errors_match_the_reference", errors_match_the_reference},
  };
  for (const auto& t : tests) {
    try {
      t.second();
      std::printf("ok   %s\n", t.first);
    } catch (const std::exception& e) {
      ++g_failures;
      std::printf("FAIL %s: %s\n", t.first, e.what());
    }
  }
  std::printf("%d failures\n", g_failures);
  return g_failures == 0 ? 0 : 1;
}
