"""Test infrastructure: mechanical g++-13 compatibility rewrite of the
reference front-end header, written to a git-ignored build folder.

silarray's include/array.h declares seven members with C++23 explicit object
parameters ("deducing this", include/array.h:353-379 and their definitions at
953-969 and 1103-1142).  g++ 13 does not implement that feature.  This script
rewrites exactly those members into const members that return T& / T* (the
non-const instantiation the reference would pick for a mutable array) and
changes nothing else.  The output goes to oracle/_ref/gen/array.h, is used only
to compile the oracle library and the reference's own doctest suite, and is
deleted by the Makefile after the build.

Usage: python oracle/patch_ref.py <reference include dir> <output file>
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
    return out


def main():
    src_dir, dst = sys.argv[1], sys.argv[2]
    with open(f"{src_dir}/array.h") as f:
        src = f.read()
    with open(dst, "w") as f:
        f.write(patch(src))


if __name__ == "__main__":
    main()
