"""Reads the C-ABI declared in include/hexel_b200.h into a signature table
(no torch, no library load: the build uses it to write gsplat/_abi_table.py,
the table the loader binds)."""

from __future__ import annotations

import re

KINDS = ("ptr", "int", "unsigned", "float", "size_t", "int32_t", "int64_t")
RETURNS = ("int", "size_t", "const char*", "void", "unsigned long long")


def arg_kind(decl: str) -> str:
    """The kind of one C argument declaration: "ptr" for pointers and
    cudaStream_t, else its scalar type."""
    decl = decl.strip()
    if "*" in decl or decl.startswith("cudaStream_t"):
        return "ptr"
    base = decl.rsplit(" ", 1)[0].replace("const ", "").strip()
    if base not in KINDS:
        raise ValueError(f"unsupported argument type in {decl!r}")
    return base


def parse_header(path: str) -> dict:
    """{name: (return type, [argument kinds])} for every HX_API function."""
    text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"HX_API\s+(int|size_t|const char\*|void|unsigned long long)\s+"
                         r"(hx_\w+)\s*\((.*?)\);",
                         text, flags=re.S):
        ret, name, args = m.group(1), m.group(2), " ".join(m.group(3).split())
        argv = [] if args in ("", "void") else [arg_kind(a) for a in args.split(",")]
        out[name] = (ret, argv)
    return out


def render_table(table: dict) -> str:
    """Python source of the table module."""
    lines = ['"""Signatures of the C-ABI of libhexel_b200.so, written by the build from',
             'include/hexel_b200.h (name: (return type, argument kinds)); do not edit."""',
             "", "SIGNATURES = {"]
    for name in sorted(table):
        ret, args = table[name]
        lines.append(f"    {name!r}: ({ret!r}, {args!r}),")
    lines.append("}")
    return "\n".join(lines) + "\n"
