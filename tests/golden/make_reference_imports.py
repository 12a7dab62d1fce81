"""Write tests/golden/reference_imports.json: every `from <module> import
<name>` in the reference's kernel/*.py whose module is one of the names the
drop-in layer aliases (flow_expert, triton_gemm, cudagraph, quant), as
[file, module, name] triples. The reference is read as text only.

    python tests/golden/make_reference_imports.py <reference checkout>
"""
import ast
import json
import os
import sys

ALIASED = ("flow_expert", "triton_gemm", "cudagraph", "quant")


def main(ref_root):
    kdir = os.path.join(ref_root, "kernel")
    out = []
    for fn in sorted(os.listdir(kdir)):
        if not fn.endswith(".py") or fn[:-3] in ALIASED:
            continue
        tree = ast.parse(open(os.path.join(kdir, fn)).read())
        for node in ast.walk(tree):
            if isinstance(node, ast.ImportFrom) and node.module in ALIASED:
                out.extend([f"kernel/{fn}", node.module, a.name] for a in node.names)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_imports.json")
    with open(path, "w") as f:
        f.write("[\n" + ",\n".join(json.dumps(t) for t in sorted(out)) + "\n]\n")
    print(f"{len(out)} imports -> {path}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_reference_imports.py <path of the reference checkout>")
    main(sys.argv[1])
