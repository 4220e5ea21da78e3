"""Golden KV plans of the LingBot runtime, generated from the reference's own ``eager_plans``
(``fastworld/models/lingbot_v2/static.py:30-46``).

The reference module imports the un-vendored LingBot package at load time, so this script
compiles only that function from the reference source (its module constants LOCAL_ATTN and SINK
come from ``engine.py:24``) and records its output for a few window shapes:

    python tests/golden/make_lingbot_plans.py /path/to/fastworld   # writes lingbot_plans.json
"""
import ast
import json
import os
import sys


def reference_eager_plans(root: str):
    src = open(os.path.join(root, "fastworld", "models", "lingbot_v2", "static.py")).read()
    fn = [n for n in ast.parse(src).body if isinstance(n, ast.FunctionDef) and n.name == "eager_plans"][0]
    ns = {"LOCAL_ATTN": 18, "SINK": 6}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "static.py", "exec"), ns)
    return ns["eager_plans"]


def main():
    root = sys.argv[1]
    ep = reference_eager_plans(root)
    cases = [(40, 4, 18, 6), (24, 3, 12, 3), (30, 2, 9, 0), (20, 4, -1, 6), (16, 4, 10, 2)]
    out = [{"n": n, "C": C, "W": W, "S": S, "plans": ep(n, C, W, S)} for n, C, W, S in cases]
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lingbot_plans.json")
    json.dump(out, open(path, "w"))
    print("wrote", path)


if __name__ == "__main__":
    main()
