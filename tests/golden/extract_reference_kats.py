"""Extracts the reference's own known answers into JSON fixtures (run in the build container only).

Sources (paths within caelunshun/ptx-std):
  - examples/tcgen05_ptxas/descriptor.rs: the compile-time `const _: () = assert!(...)` checks of
    the tcgen05 descriptor encodings (their expected values come from CUTLASS's bitfield unions and
    the PTX ISA, per that file's header). Each builder chain is rewritten from Rust syntax into a
    Python expression over the same builder names (``::`` -> ``.``, ``None`` -> ``None_``,
    ``true`` -> ``True``), so that the tests evaluate the reference's own expressions;
  - src/data_types/float8.rs, float4.rs: the named bit-pattern constants of each format with the
    value their doc comment states.

    python tests/golden/extract_reference_kats.py [/path/to/reference]

Writes tests/golden/descriptor_kats.json and tests/golden/format_constants.json.
"""

from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _pyexpr(rust: str) -> str:
    e = " ".join(rust.split())
    e = e.replace("::", ".")
    e = re.sub(r"\.None\b", ".None_", e)
    e = re.sub(r"\btrue\b", "True", e)
    e = re.sub(r"\bfalse\b", "False", e)
    e = e.replace("( ", "(").replace(" )", ")")
    return e


def extract_descriptor_kats(ref: str) -> dict:
    path = os.path.join(ref, "examples", "tcgen05_ptxas", "descriptor.rs")
    src = open(path).read()
    lines = src.split("\n")
    aliases = {}
    m = re.search(r"use ptx_std::tcgen05::\{(.*?)\};", src, re.S)
    for a, b in re.findall(r"(\w+) as (\w+)", m.group(1)):
        aliases[b] = a
    kinds = dict(re.findall(r"type (\w+) = InstrDescriptor<\{ MmaKind::(\w+) \}>;", src))

    items = []
    i = 0
    pending_cfg = None
    while i < len(lines):
        ln = lines[i].strip()
        if ln.startswith("#[cfg("):
            pending_cfg = ln
            i += 1
            continue
        start = i
        if ln.startswith("const _: () =") or re.match(r"const [A-Z0-9_]+: \w+ =", ln):
            buf = [ln]
            while not buf[-1].rstrip().endswith(";"):
                i += 1
                buf.append(lines[i].strip())
            text = " ".join(buf)
            if text.startswith("const _: () ="):
                body = text[len("const _: () ="):].strip().rstrip(";").strip()
                assert body.startswith("assert!(") and body.endswith(")"), body
                expr = body[len("assert!("):-1].strip()
                items.append({"line": start + 1, "kind": "assert", "rust": expr,
                              "expr": _pyexpr(expr), "cfg": pending_cfg})
            else:
                mm = re.match(r"const ([A-Z0-9_]+): (\w+) = (.*);$", text)
                items.append({"line": start + 1, "kind": "const", "name": mm.group(1),
                              "type": mm.group(2), "rust": mm.group(3),
                              "expr": _pyexpr(mm.group(3)), "cfg": pending_cfg})
            pending_cfg = None
        elif ln and not ln.startswith("//"):
            pending_cfg = None if not ln.startswith("#[") else pending_cfg
        i += 1
    return {"source": "examples/tcgen05_ptxas/descriptor.rs", "aliases": aliases,
            "kinds": kinds, "items": items}


_WORDS = {"Positive zero.": "0.0", "Negative zero.": "-0.0", "One.": "1.0",
          "Negative one.": "-1.0", "Positive infinity.": "inf", "Negative infinity.": "-inf",
          "A quiet NaN.": "nan"}


def _doc_value(doc: str) -> str:
    if doc in _WORDS:
        return _WORDS[doc]
    if "NaN" in doc:
        return "nan"
    m = re.search(r"\(([-0-9.^]+)\)", doc.replace("`", "").replace("2^0, encoded as 0x7f", "1"))
    if m:
        return m.group(1)
    m = re.search(r"\(`?(2\^-?\d+)`?", doc)
    if m:
        return m.group(1)
    raise ValueError(doc)


def extract_constants(ref: str) -> dict:
    out = {}
    for fname, fmts in (("float8.rs", ("f8e4m3", "f8e5m2", "f8e8m0")), ("float4.rs", ("f4e2m1",)),
                        ("float6.rs", ("f6e2m3", "f6e3m2"))):
        path = os.path.join(ref, "src", "data_types", fname)
        lines = open(path).read().split("\n")
        cur, doc = None, None
        for n, raw in enumerate(lines, 1):
            ln = raw.strip()
            m = re.match(r"(f\d\w+), width: \d+,", ln)
            if m and m.group(1) in fmts:
                cur = m.group(1)
                out.setdefault(cur, [])
                continue
            if cur and ln.startswith("///"):
                doc = ln[3:].strip()
                continue
            m = re.match(r"([A-Z_]+) = (0x[0-9A-Fa-f]+);", ln)
            if cur and m:
                out[cur].append({"name": m.group(1), "code": int(m.group(2), 16),
                                 "doc": doc, "value": _doc_value(doc), "line": n,
                                 "file": f"src/data_types/{fname}"})
                continue
            if cur and ln == "}" and out[cur]:
                cur = None
    return out


def main() -> int:
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    kats = extract_descriptor_kats(ref)
    with open(os.path.join(HERE, "descriptor_kats.json"), "w") as f:
        json.dump(kats, f, indent=1)
    consts = extract_constants(ref)
    with open(os.path.join(HERE, "format_constants.json"), "w") as f:
        json.dump(consts, f, indent=1)
    print(len(kats["items"]), "descriptor items;",
          {k: len(v) for k, v in consts.items()}, "constants")
    return 0


if __name__ == "__main__":
    sys.exit(main())
