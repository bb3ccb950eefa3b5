"""Print named top-level functions of a C/C++ source file to stdout.

Build helper for oracle/Makefile: it pulls popcorn's test-side CPU reference
loops (static functions in test/test_quantize.cu, a file that as a whole does
not compile with this container's g++) out of the reference checkout so they
can be piped straight into the compiler. Nothing it prints is written into
the repository; the only product is the compiled oracle/_ref/libref_loops.so.

usage: python3 extract_ref.py FILE NAME [NAME ...]
"""
import re
import sys


def extract(text: str, name: str) -> str:
    m = re.search(r"^static\s+void\s+" + re.escape(name) + r"\s*\(", text, re.M)
    if m is None:
        raise SystemExit(f"extract_ref: function {name!r} not found")
    start = m.start()
    open_brace = text.index("{", m.end())
    depth = 0
    for i in range(open_brace, len(text)):
        c = text[i]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return text[start : i + 1] + "\n"
    raise SystemExit(f"extract_ref: unbalanced braces in {name!r}")


def main() -> None:
    if len(sys.argv) < 3:
        raise SystemExit(__doc__)
    with open(sys.argv[1], encoding="utf-8") as f:
        text = f.read()
    for name in sys.argv[2:]:
        sys.stdout.write(extract(text, name))


if __name__ == "__main__":
    main()
