"""Search space = the plugin's variants() over its declared axes.  The pipeline only knows an
axis's name and the resources it moves (reference tempo/core/search/space.py)."""
from __future__ import annotations


def enumerate_variants(plugin, op, limit=None):
    out = []
    for h in plugin.skeletons.variants(op):
        out.append(h)
        if limit is not None and len(out) >= limit:
            break
    return out


def axes_table(plugin) -> str:
    rows = [f"SEARCH AXES DECLARED BY PLUGIN {plugin.id}"]
    for a in plugin.skeletons.axes():
        rows.append(f"  {a.name:<14} moves: {', '.join(sorted(a.affects)) or '-'}")
    return "\n".join(rows)


def touching(plugin, resource: str):
    return tuple(a.name for a in plugin.skeletons.axes() if resource in a.affects)
