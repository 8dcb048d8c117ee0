"""Test infrastructure: mechanical g++-13 compatibility rewrite of the
reference front-end header, written to a git-ignored build folder.

silarray's include/array.h declares seven members with C++23 explicit object
parameters ("deducing this", include/array.h:353-379 and their definitions at
953-969 and 1103-1142).  g++ 13 does not implement that feature.  This script
rewrites exactly those members into const members that return T& / T* (the
non-const instantiation the reference would pick for a mutable array).

One defect fix as well: after evaluating a graph, array<T>::evaluate_node_
and sil::eval (include/array.h:1973-1985, 2835-2888) clear the `visited` flag
of every node in the topological order, but evaluating a node releases its
inputs (array.h:2059-2060), so intermediate nodes nobody else holds are
already freed: the clearing loop writes into freed memory (AddressSanitizer:
heap-use-after-free at array.h:2881), which corrupted the heap in silarray's
own bench_transformer.cpp on this backend.  The rewrite clears the flags
right after the topological sort instead (they are only read by the sort),
which changes nothing else.  The output goes to oracle/_ref/gen/array.h, is used only
to compile the oracle library and the reference's own doctest suite, and is
deleted by the Makefile after the build.

With --dropin (the builds on the B200 backend headers only, never the CPU
reference build): sum(axis) for every axis but 0 of a 2-D array runs the
reference's own loop on the host even in GPU mode (include/array.h:2303-2317);
the drop-in build routes dense inputs to gpu::sum_axis_f32, which adds in the
same order on the GPU up to 4096 terms per output (bit-identical results).

Usage: python oracle/patch_ref.py <reference include dir> <output file> [--dropin]
"""
import re
import sys


def patch(src: str) -> str:
    out = src
    # In-class declarations (include/array.h:353-379).
    decls = [
        ("auto *buffer_data(this auto &&self);", "T *buffer_data() const;"),
        ("auto buffer_span(this auto &&self);", "std::span<T> buffer_span() const;"),
        ("auto &at(this auto &&self);", "T &at() const;"),
        ("auto &at(this auto &&self, size_t i);", "T &at(size_t i) const;"),
        ("auto &operator[](this auto &&self, size_t x, size_t y);",
         "T &operator[](size_t x, size_t y) const;"),
        ("auto &operator[](this auto &&self, size_t x, size_t y, size_t z);",
         "T &operator[](size_t x, size_t y, size_t z) const;"),
        ("auto &at(this auto &&self, const std::vector<size_t> &position);",
         "T &at(const std::vector<size_t> &position) const;"),
    ]
    for a, b in decls:
        if a not in out:
            raise SystemExit(f"patch_ref: declaration not found: {a}")
        out = out.replace(a, b)

    # Out-of-class definitions: rewrite the signature and bind `self`.
    bind = " auto &self = const_cast<array &>(*this);"
    pat = re.compile(
        r"inline auto (\*|&)?\s*array<T>::(buffer_data|buffer_span|at|operator\[\])"
        r"\(this auto &&self(,\s*)?([^)]*)\)\s*\{",
        re.S,
    )

    def repl(m):
        ret = {"*": "T *", "&": "T &", None: "std::span<T> "}[m.group(1)]
        args = m.group(4).strip()
        return f"inline {ret}array<T>::{m.group(2)}({args}) const {{{bind}"

    out, n = pat.subn(repl, out)
    if n != 7:
        raise SystemExit(f"patch_ref: expected 7 definitions, rewrote {n}")
    if "this auto" in out:
        raise SystemExit("patch_ref: an explicit object parameter is left")

    # The visited-flag reset, moved ahead of the evaluation loops.
    a = ("  auto order = topo_sort_({node.get()});\n\n"
         "  for (auto *cur : order) {\n"
         "    if (cur->evaluated) continue;\n"
         "    evaluate_single_node_(cur);\n"
         "  }\n\n"
         "  for (auto *cur : order) cur->visited = false;\n")
    b = ("  auto order = topo_sort_({node.get()});\n"
         "  for (auto *cur : order) cur->visited = false;\n\n"
         "  for (auto *cur : order) {\n"
         "    if (cur->evaluated) continue;\n"
         "    evaluate_single_node_(cur);\n"
         "  }\n")
    if out.count(a) != 1:
        raise SystemExit("patch_ref: evaluate_node_ loop not found")
    out = out.replace(a, b)
    a = ("  for (auto *cur : order) {\n"
         "    if (cur->evaluated) continue;\n"
         "    array<float>::evaluate_single_node_(cur);\n"
         "  }\n")
    c = "  for (auto *cur : order) cur->visited = false;\n\n  // Sync storage"
    if out.count(a) != 1 or out.count(c) != 1:
        raise SystemExit("patch_ref: sil::eval loops not found")
    out = out.replace(c, "  // Sync storage")
    out = out.replace(a, "  for (auto *cur : order) cur->visited = false;\n" + a)
    return out


DROPIN_SUM_AXIS_FROM = """        } else {
          input.enumerate_position_([&](const auto &pos) {
            auto p = pos;
            p.erase(p.begin() + axis);
            tmp.at(p) += input.at(pos);
          });
        }
        store_result(tmp);"""

DROPIN_SUM_AXIS_TO = """        } else if (device_ == Device::MPS && input.buffer_element_count() == input.element_count()) {
          size_t outer = 1, inner = 1;
          for (size_t d = 0; d < axis; d++) outer *= in_shape[d];
          for (size_t d = axis + 1; d < in_shape.size(); d++) inner *= in_shape[d];
          gpu::sum_axis_f32(input.storage_, tmp.storage_, outer, in_shape[axis], inner);
        } else {
          input.enumerate_position_([&](const auto &pos) {
            auto p = pos;
            p.erase(p.begin() + axis);
            tmp.at(p) += input.at(pos);
          });
        }
        store_result(tmp);"""


def patch_dropin(src: str) -> str:
    if src.count(DROPIN_SUM_AXIS_FROM) != 1:
        raise SystemExit("patch_ref: sum(axis) host loop not found")
    return src.replace(DROPIN_SUM_AXIS_FROM, DROPIN_SUM_AXIS_TO)


def main():
    src_dir, dst = sys.argv[1], sys.argv[2]
    with open(f"{src_dir}/array.h") as f:
        src = f.read()
    out = patch(src)
    if "--dropin" in sys.argv[3:]:
        out = patch_dropin(out)
    with open(dst, "w") as f:
        f.write(out)


if __name__ == "__main__":
    main()
