"""Extracts the reference's known-answer vectors into reference_kat.json.

Reads the unit tests of ZeroR0R/tensor-inference-runtime as text (they are the
only golden vectors the reference has for this path; its golden-token tests
need a model file that is not distributed) and writes the arrays and expected
values they assert.  Run from the repo root, giving the directory of a checkout
of the reference crate:

    python tests/golden/extract_kat.py REFERENCE_CHECKOUT

The tests read the committed JSON; nothing reads the reference at test time.
"""
import json
import os
import re
import sys


def _block(src, start_pat, open_ch="[", close_ch="]"):
    i = src.index(start_pat)
    j = src.index(open_ch, i)
    depth = 0
    for k in range(j, len(src)):
        if src[k] == open_ch:
            depth += 1
        elif src[k] == close_ch:
            depth -= 1
            if depth == 0:
                return src[j + 1:k]
    raise ValueError(start_pat)


def _nums(text, cast=float):
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"(?<=\d)_(?=\d)", "", text)
    return [cast(t.replace("_", "")) for t in re.findall(r"-?\d[\d_]*(?:\.\d+)?(?:e-?\d+)?", text)]


def _fn_body(src, name):
    i = src.index(f"fn {name}")
    return src[i:src.index("\n}", i)]


def main(ref):
    math_rs = open(os.path.join(ref, "src/math.rs")).read()
    kern_rs = open(os.path.join(ref, "src/kernels.rs")).read()
    tok_rs = open(os.path.join(ref, "src/tokenizer.rs")).read()

    kat = {"source": "ZeroR0R/tensor-inference-runtime unit tests", "cases": {}}
    c = kat["cases"]

    # src/kernels.rs:37-55 test_output_first_block
    body = _fn_body(kern_rs, "test_output_first_block")
    c["activated_q8_first_block"] = {
        "cite": "src/kernels.rs:37-55",
        "input_value": _nums(re.search(r"vec!\[([^;]+);", body).group(1))[0],
        "input_len": int(re.search(r"vec!\[[^;]+;\s*(\d+)\]", body).group(1)),
        "expected_first_block": _nums(_block(body, "let expected"), int),
    }

    # src/math.rs:248-255 dot_product_test
    body = _fn_body(math_rs, "dot_product_test")
    vecs = re.findall(r"vec!\[([^\]]+)\]", body)
    c["dot_prod_f32"] = {"cite": "src/math.rs:248-255", "a": _nums(vecs[0]), "b": _nums(vecs[1]),
                         "expected": _nums(re.search(r"product: f32 = ([^;]+);", body).group(1))[0]}

    # src/math.rs:286-345 q8_dequant_test
    body = _fn_body(math_rs, "q8_dequant_test")
    c["q8_dequant_block"] = {
        "cite": "src/math.rs:286-345",
        "raw_block": _nums(_block(body, "let _raw_byte_block"), int),
        "scale": _nums(re.search(r"let scale = ([^;]+);", body).group(1))[0],
        "quantized": _nums(_block(body, "let quantized_int8_vals"), int),
        "dequantized": _nums(_block(body, "let dequantized_vals")),
        "tolerance": 1e-6,
    }

    # src/math.rs:347-357 dot_prod_q8_test: block of scale 1.0, weights i, a = 2.0
    body = _fn_body(math_rs, "dot_prod_q8_test")
    c["dot_prod_q8"] = {"cite": "src/math.rs:347-357", "scale": 1.0, "weights": list(range(32)),
                        "a_value": 2.0,
                        "expected": _nums(re.search(r"&block\), ([^)]+)\)", body).group(1))[0]}

    # src/math.rs:359-379 q8_matmul_test: two rows of 64 (two blocks each)
    c["q8_matmul"] = {"cite": "src/math.rs:359-379",
                      "w1": [i - 16 for i in range(32)], "w2": [8 - i for i in range(32)],
                      "blocks": [[0.5, "w1"], [0.25, "w2"], [1.5, "w2"], [2.0, "w1"]],
                      "a": [i / 16.0 - 2.0 for i in range(64)], "tolerance": 1e-4}

    # src/math.rs:381-389 rms_norm_test
    body = _fn_body(math_rs, "rms_norm_test")
    vecs = re.findall(r"vec!\[([^\]]+)\]", body)
    c["rmsnorm"] = {"cite": "src/math.rs:381-389", "a": _nums(vecs[0]), "w": _nums(vecs[1]),
                    "expected": _nums(_block(body, "let expected")), "tolerance": 1e-5}

    # src/math.rs:391-411 softmax_test
    body = _fn_body(math_rs, "softmax_test")
    c["softmax"] = {"cite": "src/math.rs:391-411",
                    "x": _nums(re.search(r"u_flat = vec!\[([^\]]+)\]", body).group(1)),
                    "expected": _nums(_block(body, "let expected")), "tolerance": 1e-6}

    # src/math.rs:413-430 rope_test
    body = _fn_body(math_rs, "rope_test")
    c["rope"] = {"cite": "src/math.rs:413-430",
                 "query": _nums(re.search(r"query = vec!\[([^\]]+)\]", body).group(1)),
                 "key": _nums(re.search(r"key: Vec<f32> = vec!\[([^\]]+)\]", body).group(1)),
                 "pos": int(re.search(r"let pos = (\d+);", body).group(1)),
                 "dim": int(re.search(r"let dim = (\d+);", body).group(1)),
                 "base": _nums(re.search(r"let base: f32 = ([^;]+);", body).group(1))[0],
                 "expected": _nums(_block(body, "let expected")), "tolerance": 1e-4}

    # src/tokenizer.rs:237-240 sample_test
    body = _fn_body(tok_rs, "sample_test")
    m = re.search(r"sample\(&\[([^\]]+)\]\), (\d+)\)", body)
    c["sample"] = {"cite": "src/tokenizer.rs:237-240", "logits": _nums(m.group(1)),
                   "expected": int(m.group(2))}

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kat.json")
    with open(out, "w") as f:
        json.dump(kat, f, indent=1)
    print(out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: extract_kat.py REFERENCE_CHECKOUT  (the reference crate's root directory)")
    main(sys.argv[1])
