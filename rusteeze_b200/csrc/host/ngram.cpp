// N-gram (prompt-lookup) draft proposals for speculative decoding.
//
// The reference's speculative configuration names an n-gram proposer next to draft and
// Medusa models (crates/rusteeze-core/src/config.rs:602-646) but never implements one.
// Here, for each sequence (prompt + generated tokens so far): take its last n tokens,
// for n from n_max down to n_min; find the most recent earlier position where those n
// tokens occur; propose the (up to) k tokens that followed them there.  The longest
// suffix that recurs wins; a sequence with no recurring suffix gets no proposal.
//
// The search runs for every decoding sequence on every speculative step, so it is a
// tight C++ loop over the token buffer (first-token filter, then an n-token compare),
// with the GIL released, rather than Python or NumPy.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <vector>

namespace py = pybind11;

namespace {

// Writes up to k proposed tokens for one sequence into out; returns how many.
int propose_one(const int64_t* t, int64_t L, int k, int n_max, int n_min, int64_t* out) {
  if (L < 2 || k <= 0) return 0;
  const int top = static_cast<int>(std::min<int64_t>(n_max, L - 1));
  for (int n = top; n >= n_min; --n) {
    const int64_t* pat = t + (L - n);
    // candidate starts i with i + n <= L - 1 (a continuation token exists), latest first
    for (int64_t i = L - n - 1; i >= 0; --i) {
      if (t[i] != pat[0]) continue;
      int j = 1;
      while (j < n && t[i + j] == pat[j]) ++j;
      if (j < n) continue;
      const int64_t from = i + n;
      const int cnt = static_cast<int>(std::min<int64_t>(k, L - from));
      for (int c = 0; c < cnt; ++c) out[c] = t[from + c];
      return cnt;
    }
  }
  return 0;
}

// tokens: one int64 array per sequence.  Returns (proposals [S, k] int64, padded with the
// sequence's last token; counts [S] int32).
py::tuple ngram_propose(const std::vector<py::array_t<int64_t, py::array::c_style | py::array::forcecast>>& tokens,
                        int k, int n_max, int n_min) {
  if (k < 1 || n_min < 1 || n_max < n_min) throw std::invalid_argument("need k >= 1 and 1 <= n_min <= n_max");
  const size_t S = tokens.size();
  py::array_t<int64_t> props({static_cast<py::ssize_t>(S), static_cast<py::ssize_t>(k)});
  py::array_t<int32_t> counts(static_cast<py::ssize_t>(S));
  std::vector<const int64_t*> ptr(S);
  std::vector<int64_t> len(S);
  for (size_t s = 0; s < S; ++s) {
    if (tokens[s].ndim() != 1) throw std::invalid_argument("token arrays must be 1-D");
    ptr[s] = tokens[s].data();
    len[s] = tokens[s].shape(0);
  }
  int64_t* P = props.mutable_data();
  int32_t* C = counts.mutable_data();
  {
    py::gil_scoped_release nogil;
    for (size_t s = 0; s < S; ++s) {
      int64_t* row = P + s * k;
      const int c = propose_one(ptr[s], len[s], k, n_max, n_min, row);
      const int64_t pad = c > 0 ? row[c - 1] : (len[s] > 0 ? ptr[s][len[s] - 1] : 0);
      for (int i = c; i < k; ++i) row[i] = pad;
      C[s] = c;
    }
  }
  return py::make_tuple(props, counts);
}

}  // namespace

void bind_ngram(py::module_& m) {
  m.def("ngram_propose", &ngram_propose, py::arg("tokens"), py::arg("k"), py::arg("n_max"), py::arg("n_min"),
        "Prompt-lookup proposals: (int64 [S, k] tokens padded with the last token, int32 [S] counts)");
}
