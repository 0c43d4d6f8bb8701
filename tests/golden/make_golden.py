"""Extract the known-answer vectors of the reference's own tests into JSON fixtures.

The reference (liuy/wukong) pins its CUDA ops with hand-written vectors in two
test files: the gtest suite ``test_cuda.cu`` and the Go suite
``llm/array_test.go``.  This script reads both files as plain text, pulls out
every literal array per test, and writes ``tests/golden/reference_kat.json``.
Nothing from the reference is executed.

Usage (in a checkout that has the reference sources mounted):

    python tests/golden/make_golden.py <reference checkout>

(default: $WUKONG_REFERENCE_SRC, else /root/reference)

The JSON maps ``"<suite>/<test>" -> {"<array name>": [values...]}``.  For Go
tests that build tensors inline (``x, err := MakeTensorErr(Shape{..}, []float32{..})``)
the array is stored under the variable name; bare slice literals
(``expected := []float32{..}``) under their own name.  Repeated names inside one
test get a numeric suffix in order of appearance (``expected``, ``expected_1``).
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _numbers(body):
    body = re.sub(r"//[^\n]*", "", body)
    out = []
    for tok in re.split(r"[,\s]+", body):
        tok = tok.strip().rstrip("f").rstrip("F")
        if not tok:
            continue
        v = float(tok)
        out.append(int(v) if re.fullmatch(r"-?\d+", tok) else v)
    return out


def _blocks(text, opener):
    """Yield (name, body) for each top-level test block starting with `opener`."""
    for m in re.finditer(opener, text):
        name = m.group(1)
        start = text.index("{", m.end() - 1)
        depth, i = 0, start
        while True:
            c = text[i]
            if c == "{":
                depth += 1
            elif c == "}":
                depth -= 1
                if depth == 0:
                    break
            i += 1
        yield name, text[start + 1:i]


def _put(d, name, vals):
    key, n = name, 1
    while key in d:
        key = f"{name}_{n}"
        n += 1
    d[key] = vals


def parse_cpp(path):
    text = open(path).read()
    tests = {}
    arr = re.compile(r"(?:float|int|uint8_t)\s+(\w+)\s*\[[^\]]*\]\s*=\s*\{(.*?)\};", re.S)
    for name, body in _blocks(text, r"TEST\(Cuda,\s*(\w+)\)\s*\{"):
        d = {}
        for m in arr.finditer(body):
            _put(d, m.group(1), _numbers(m.group(2)))
        tests[f"test_cuda.cu/{name}"] = d
    return tests


def parse_go(path):
    text = open(path).read()
    tests = {}
    make = re.compile(r"(\w+),\s*err\s*:?=\s*MakeTensorErr\(Shape\{[^}]*\},\s*\[\]\w+\{(.*?)\}\)", re.S)
    lit = re.compile(r"(\w+)\s*:?=\s*\[\](?:float32|int32|int16|uint8)\{(.*?)\}", re.S)
    field = re.compile(r"(\w+):\s*\[\](?:float32|int32|int16|uint8)\{(.*?)\}", re.S)
    for name, body in _blocks(text, r"func\s+(Test\w+)\(t \*testing\.T\)\s*\{"):
        d = {}
        # commented-out code is not a vector
        clean = "\n".join(l for l in body.splitlines() if not l.strip().startswith("//"))
        for rx in (make, lit, field):
            for m in rx.finditer(clean):
                _put(d, m.group(1), _numbers(m.group(2)))
        tests[f"array_test.go/{name}"] = d
    return tests


def main(ref):
    out = {}
    out.update(parse_cpp(os.path.join(ref, "test_cuda.cu")))
    out.update(parse_go(os.path.join(ref, "llm", "array_test.go")))
    dst = os.path.join(HERE, "reference_kat.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print(f"wrote {dst}: {len(out)} tests")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("WUKONG_REFERENCE_SRC", "/root/reference"))
