"""Reports of accuracy comparisons without plotting libraries (the reference renders KV / logit
comparisons with plotly: ``accuracy/kv_cache_visualize.py`` ``export_html_report`` ``:103``,
``export_json`` ``:237``; ``logit_visualization.py``; ``plotting.py``).  Here a report is a JSON
document plus a self-contained HTML page: one table row per compared tensor, with an inline bar
for its relative error, so it opens in any browser of an air-gapped machine."""

from __future__ import annotations

import dataclasses
import html
import json
import math


def _rows(results) -> list[dict]:
    out = []
    for r in results:
        out.append(dataclasses.asdict(r) if dataclasses.is_dataclass(r) else dict(r))
    return out


def export_json(results, path: str, meta: dict | None = None) -> None:
    with open(path, "w") as f:
        json.dump({"meta": meta or {}, "results": _rows(results)}, f, indent=1, default=str)


def export_html(results, path: str, title: str = "accuracy report", metric: str = "rel_l2") -> None:
    """HTML table of the results (dataclasses or dicts); ``metric`` drives the bar length on a
    log scale from 1e-6 to 1."""
    rows = _rows(results)
    cols = list(rows[0].keys()) if rows else []
    body = []
    for r in rows:
        v = r.get(metric)
        frac = 0.0
        if isinstance(v, (int, float)) and v > 0:
            frac = min(1.0, max(0.0, (math.log10(v) + 6) / 6))
        color = "#c33" if r.get("passed") is False else "#3a3"
        cells = "".join(f"<td>{html.escape(f'{r[c]:.4g}' if isinstance(r[c], float) else str(r[c]))}</td>"
                        for c in cols)
        bar = f'<td><div style="background:{color};height:10px;width:{int(200 * frac)}px"></div></td>'
        body.append(f"<tr>{cells}{bar}</tr>")
    head = "".join(f"<th>{html.escape(c)}</th>" for c in cols) + f"<th>{html.escape(metric)} (log)</th>"
    doc = (f"<!doctype html><html><head><meta charset='utf-8'><title>{html.escape(title)}</title>"
           "<style>td,th{padding:2px 8px;font:12px monospace;text-align:right}</style></head>"
           f"<body><h3>{html.escape(title)}</h3><table><tr>{head}</tr>{''.join(body)}</table></body></html>")
    with open(path, "w") as f:
        f.write(doc)
