"""Generate tests/golden/linear_fallback.pt by running the REFERENCE's own code (not a restatement).

The reference's ComfyUI node (comfyui/custom_nodes/comfyui_xdna1_npu/__init__.py) replaces nn.Linear.forward with
_npu_linear_forward (:146-158); with no NPU runtime present it takes its CPU fallback F.linear(x, weight, bias)
(:150-151). That fallback is the reference's CPU semantics for the GEMM, so its outputs on seeded bf16-valued inputs
pin the oracle (oracle.linear_ref). The module imports only numpy and torch at top level, so it loads here even
though the NPU stack (aie.iron, pyxrt) is absent.

Run where the reference tree is available:  python tests/golden/make_golden.py <reference_root>
"""
import importlib.util
import os
import sys

import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "linear_fallback.pt")
# (M, K, N): the reference test's unaligned case (scripts/05-gemm-test.py:18) and small SD1.5-like shapes.
SHAPES = [(100, 100, 100), (77, 320, 320), (20, 768, 64), (33, 640, 136), (5, 1280, 64)]


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference_root>")
    node_file = os.path.join(sys.argv[1], "comfyui", "custom_nodes", "comfyui_xdna1_npu", "__init__.py")
    spec = importlib.util.spec_from_file_location("reference_xdna1_node", node_file)
    node = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(node)
    assert node._RUNTIME is None, "the fallback path needs no NPU runtime"
    cases = []
    for i, (M, K, N) in enumerate(SHAPES):
        g = torch.Generator().manual_seed(1000 + i)
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
        lin = torch.nn.Linear(K, N)
        with torch.no_grad():
            lin.weight.copy_(w.float())
            lin.bias.copy_(b.float())
        y = node._npu_linear_forward(lin, x.float()).detach()   # the reference's own forward → its CPU fallback
        cases.append({"M": M, "K": K, "N": N, "x": x, "w": w, "b": b, "y": y})
    torch.save({"source": "comfyui/custom_nodes/comfyui_xdna1_npu/__init__.py:_npu_linear_forward (CPU fallback)",
                "cases": cases}, OUT)
    print(f"wrote {OUT} ({len(cases)} cases)")


if __name__ == "__main__":
    main()
