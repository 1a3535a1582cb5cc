"""Text drawings of a recorded graph: Graphviz DOT and Mermaid flowchart source (the
reference's viz.py; the same output format, so drawings and tests carry over).

Tensors are listed inputs first (post-order from the outputs); leaves that require grad are
drawn shaded, other leaves dashed, ops as rounded boxes with their name and output shape,
outputs with a heavier outline. Only the host-side graph is read, no device data. A backward
pass without ``retain_graph`` releases the nodes it walks, so draw before it.
"""

from __future__ import annotations

from collections.abc import Iterable, Mapping
from typing import Literal, NamedTuple

from tensorgrad_b200.tensor import Tensor

__all__ = ["to_dot", "to_mermaid"]

Direction = Literal["TB", "LR"]

_PARAM_FILL, _OP_FILL, _EDGE, _INK, _MUTED = "#dfeafa", "#f3f2ee", "#898781", "#0b0b0b", "#898781"


class _Item(NamedTuple):
    key: str
    title: str
    shape: str
    kind: str  # "param", "constant" or "op"
    is_output: bool


def _walk(roots: Iterable[Tensor], names: Mapping[str, Tensor] | None
          ) -> tuple[list[_Item], list[tuple[str, str]]]:
    outputs = list(roots)
    if not outputs:
        raise ValueError("pass at least one tensor to draw")
    label = {id(t): n for n, t in (names or {}).items()}
    out_ids = {id(t) for t in outputs}
    ordered: list[Tensor] = []
    seen: set[int] = set()
    todo: list[tuple[Tensor, bool]] = [(t, False) for t in reversed(outputs)]
    while todo:
        t, done = todo.pop()
        if done:
            ordered.append(t)
        elif id(t) not in seen:
            seen.add(id(t))
            todo.append((t, True))
            if t._node is not None:
                todo.extend((p, False) for p in reversed(t._node.parents))
    key = {id(t): f"n{i}" for i, t in enumerate(ordered)}
    items: list[_Item] = []
    edges: list[tuple[str, str]] = []
    for t in ordered:
        name = label.get(id(t))
        shape = "scalar" if t.ndim == 0 else str(t.shape)
        if t._node is None:
            kind = "param" if t.requires_grad else "constant"
            title = name or ("input" if t.requires_grad else "constant")
        else:
            kind = "op"
            title = t._node.op if name is None else f"{name} = {t._node.op}"
            parents = list(dict.fromkeys(key[id(p)] for p in t._node.parents))
            edges.extend((p, key[id(t)]) for p in parents)
        items.append(_Item(key[id(t)], title, shape, kind, id(t) in out_ids))
    return items, edges


def to_dot(*tensors: Tensor, names: Mapping[str, Tensor] | None = None,
           direction: Direction = "TB") -> str:
    """Graphviz DOT source of the graph behind ``tensors``; ``names`` labels tensors (e.g.
    ``dict(model.named_parameters())``), ``direction`` is ``"TB"`` or ``"LR"``."""
    items, edges = _walk(tensors, names)
    out = ["digraph tensorgrad {", f"  rankdir={direction};",
           f'  node [fontname="Helvetica", fontsize=10, color="{_EDGE}", fontcolor="{_INK}"];',
           f'  edge [color="{_EDGE}", arrowsize=0.6];']
    styles = {"param": f'shape=box, style="filled", fillcolor="{_PARAM_FILL}"',
              "constant": f'shape=box, style="dashed", fontcolor="{_MUTED}"',
              "op": f'shape=box, style="rounded,filled", fillcolor="{_OP_FILL}"'}
    for it in items:
        text = f"{it.title}\\n{it.shape}".replace('"', '\\"')
        style = styles[it.kind] + (", penwidth=2" if it.is_output else "")
        out.append(f'  {it.key} [label="{text}", {style}];')
    out += [f"  {a} -> {b};" for a, b in edges]
    out.append("}")
    return "\n".join(out) + "\n"


def to_mermaid(*tensors: Tensor, names: Mapping[str, Tensor] | None = None,
               direction: Direction = "TB") -> str:
    """Mermaid flowchart source of the graph behind ``tensors`` (arguments as
    :func:`to_dot`)."""
    items, edges = _walk(tensors, names)
    out = [f"flowchart {direction}"]
    for it in items:
        text = f"{it.title}<br/>{it.shape}".replace('"', "#quot;")
        if it.is_output:
            left, right = "([", "])"
        elif it.kind == "op":
            left, right = "(", ")"
        else:
            left, right = "[", "]"
        out.append(f'    {it.key}{left}"{text}"{right}:::{it.kind}')
    out += [f"    {a} --> {b}" for a, b in edges]
    out += [f"    classDef param fill:{_PARAM_FILL},stroke:{_EDGE},color:{_INK}",
            f"    classDef constant fill:none,stroke:{_EDGE},stroke-dasharray:4 3,color:{_MUTED}",
            f"    classDef op fill:{_OP_FILL},stroke:{_EDGE},color:{_INK}"]
    return "\n".join(out) + "\n"
