"""Print a string constant assigned at module level in a Python file, without
running the file — TEST INFRASTRUCTURE (oracle/Makefile, target `ref`).

The reference's CUTLASS depthwise variants keep their CUDA source in
``_CUDA_SOURCE = r\"\"\"...\"\"\"`` inside
data/depthwise_conv_7x7_cuda/model_cutlass*.py and JIT-build it on import;
importing would start that build, so the constant is read from the syntax
tree instead and compiled by the Makefile, unmodified, for sm_100a.

    python extract_ref_source.py <file.py> <NAME> > out.cu
"""
import ast
import sys


def main(path: str, name: str) -> int:
    tree = ast.parse(open(path).read(), filename=path)
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == name for t in node.targets):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                sys.stdout.write(node.value.value)
                return 0
    print(f"{name} not found in {path}", file=sys.stderr)
    return 1


if __name__ == "__main__":
    sys.exit(main(sys.argv[1], sys.argv[2]))
