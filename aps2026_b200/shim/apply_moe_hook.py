"""Applies the MoE part of the drop-in to the reference's src/tensor.cu.

moe_forward_grouped_gpu (ezzy0654/aps2026 src/tensor.cu:2790-2928) launches
the reference's private expert GEMMs, so it stays in tensor.cu; only two
parts of its body change:

  routing   the scratch memsets, k_moe_top2, k_moe_offsets_work and
            k_moe_fill_stable (:2804-2821) become one call of
            b2_dropin::moe_route (b2_moe_route over the C ABI);
  combine   the k_moe_combine launch (:2922-2926) becomes one call of
            b2_dropin::moe_combine (b2_moe_combine).

Both write the reference's own MoeScratch buffers and output tensor, in the
formats its grouped GEMMs read. The hooks are declared in moe_hook.h and
defined in tensor_ops_b2.cu.

Usage: python apply_moe_hook.py SRC_TENSOR_CU OUT_CU

The source is read, never modified. Each replaced span is located by the
kernel names it launches and must be found exactly once inside the function
(the script fails otherwise, rather than guess at a changed source).
"""
from __future__ import annotations

import re
import sys

ROUTE_CALL = (
    "b2_dropin::moe_route(router.cuda_data(), rows, scratch.routes, scratch.counts, scratch.offsets,\n"
    "                         scratch.assignment_rows, scratch.route_positions, scratch.work_expert,\n"
    "                         scratch.work_start, scratch.work_expert_tall, scratch.work_start_tall);\n"
)
COMBINE_CALL = (
    "b2_dropin::moe_combine(expert_output.cuda_data(), assignments, scratch.routes,\n"
    "                           scratch.route_positions, out.cuda_data_write(), rows, h);\n"
)
ROUTING_KERNELS = ("k_moe_top2", "k_moe_offsets_work", "k_moe_fill_stable")


def _function_body(src: str, name: str) -> tuple[int, int]:
    """[start, end) of the body braces of the definition of `name`."""
    m = re.search(r"\bvoid\s+" + name + r"\s*\([^;{]*\)\s*\{", src)
    if not m:
        raise SystemExit(f"apply_moe_hook: definition of {name} not found")
    depth, i = 0, m.end() - 1
    while i < len(src):
        depth += {"{": 1, "}": -1}.get(src[i], 0)
        i += 1
        if depth == 0:
            return m.end() - 1, i
    raise SystemExit(f"apply_moe_hook: unbalanced braces in {name}")


def _statement_end(text: str, pos: int) -> int:
    """Index just past the ';' that ends the statement containing pos
    (parentheses balanced)."""
    depth = 0
    for i in range(pos, len(text)):
        c = text[i]
        if c == "(":
            depth += 1
        elif c == ")":
            depth -= 1
        elif c == ";" and depth == 0:
            return i + 1
    raise SystemExit("apply_moe_hook: statement without an end")


def _line_start(text: str, pos: int) -> int:
    return text.rfind("\n", 0, pos) + 1


def _once(body: str, needle: str) -> int:
    n = body.count(needle)
    if n != 1:
        raise SystemExit(f"apply_moe_hook: expected one '{needle}' in moe_forward_grouped_gpu, found {n}")
    return body.index(needle)


def patch(src: str) -> str:
    b0, b1 = _function_body(src, "moe_forward_grouped_gpu")
    body = src[b0:b1]
    # routing: from the first scratch memset through the stable fill launch
    first = body.find("cudaMemsetAsync(")
    fill = _once(body, "k_moe_fill_stable<<<")
    if first < 0 or first > fill:
        raise SystemExit("apply_moe_hook: scratch memsets not found before the routing kernels")
    r0, r1 = _line_start(body, first), _statement_end(body, fill)
    span = body[r0:r1]
    launches = re.findall(r"(\w+)\s*<<<", span)
    if tuple(launches) != ROUTING_KERNELS:
        raise SystemExit(f"apply_moe_hook: routing span launches {launches}, expected {list(ROUTING_KERNELS)}")
    indent = re.match(r"[ \t]*", body[r0:]).group(0)
    body = body[:r0] + indent + ROUTE_CALL.rstrip("\n").replace("\n  ", "\n" + indent + "  ") + body[r1:]
    # combine: the k_moe_combine launch statement
    c = _once(body, "k_moe_combine<<<")
    c0, c1 = _line_start(body, c), _statement_end(body, c)
    indent = re.match(r"[ \t]*", body[c0:]).group(0)
    body = body[:c0] + indent + COMBINE_CALL.rstrip("\n").replace("\n  ", "\n" + indent + "  ") + body[c1:]
    return '#include "moe_hook.h"\n' + src[:b0] + body + src[b1:]


def main(argv: list[str]) -> int:
    if len(argv) != 3:
        print(__doc__.strip().splitlines()[-4], file=sys.stderr)
        return 2
    with open(argv[1]) as f:
        out = patch(f.read())
    with open(argv[2], "w") as f:
        f.write(out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv))
