"""Evidence bundles: the JSON records this repository's benches and harnesses write, rendered
as markdown, CSV and one self-contained HTML page with inline SVG charts, plus scaling
figures computed from bench lines taken at several GPU counts.

Record kinds, recognised by their keys:

* ``bench``          -- a ``bench.py`` line (``metric`` + ``value``);
* ``contract``       -- a ``validate-run`` result (``contract`` + ``results``);
* ``strategy``       -- a stage-ring strategy decision (``scores`` + ``selected``);
* ``wan``            -- stage-ring WAN evidence (``name == "stage_ring_wan"`` + ``rows``);
* ``loopback``       -- a loopback-matrix row (``workers`` + ``concurrency``);
* ``real_loopback``  -- a real-checkpoint loopback report (``reference_tokens``);
* ``expert_backend`` -- a row of the expert-backend comparison (``backend`` + ``ms_per_forward``);
* ``other``          -- anything else (shown as JSON).

Scaling (``scaling_rows``): bench lines of one implementation, model and dtype at several GPU
counts give, per count, the gain over the smallest count, the efficiency (gain divided by the
GPU-count ratio: 1.0 is linear) and the marginal tokens/s per added GPU.
``capacity_efficiency`` divides an observed pipeline throughput by its ideal, the slowest
stage's service capacity.

Reference: si/experiments/reporting.py (self-contained HTML report), si/experiments/charts.py
(charts; drawn here as inline SVG, since no plotting library is installed) and
si/experiments/scaling.py (gain, marginal throughput, homogeneous and capacity-normalised
efficiency, predicted ideal throughput).
"""
from __future__ import annotations

import csv
import html
import io
import json
from pathlib import Path

KINDS = ("bench", "contract", "strategy", "wan", "loopback", "real_loopback", "expert_backend",
         "other")


def kind(rec) -> str:
    if not isinstance(rec, dict):
        return "other"
    if "metric" in rec and "value" in rec:
        return "bench"
    if "results" in rec and "contract" in rec:
        return "contract"
    if "scores" in rec and "selected" in rec:
        return "strategy"
    if rec.get("name") == "stage_ring_wan" and "rows" in rec:
        return "wan"
    if "concurrency" in rec and "workers" in rec:
        return "loopback"
    if "reference_tokens" in rec and "tokens" in rec:
        return "real_loopback"
    if "backend" in rec and "ms_per_forward" in rec:
        return "expert_backend"
    return "other"


def load(paths) -> list:
    """Records from JSON files (an object or a list of them), JSON-lines files, or logs whose
    lines starting with ``{`` are records."""
    records = []
    for path in paths:
        text = Path(path).read_text()
        try:
            doc = json.loads(text)
            records += doc if isinstance(doc, list) else [doc]
        except ValueError:
            for line in text.splitlines():
                line = line.strip()
                if line.startswith("{"):
                    try:
                        records.append(json.loads(line))
                    except ValueError:
                        pass
    return records


# ---------------------------------------------------------------------------------- scaling
def scaling_rows(records) -> list[dict]:
    """Per (impl, model, dtype) group of bench lines with at least two GPU counts: one row
    per count with ``gain``, ``efficiency`` and ``marginal_per_gpu`` against the smallest."""
    groups: dict[tuple, dict[int, dict]] = {}
    for r in records:
        if kind(r) != "bench" or not isinstance(r.get("value"), (int, float)):
            continue
        key = (r.get("impl", "ours"), (r.get("config") or {}).get("model", "-"), r.get("dtype", "-"))
        groups.setdefault(key, {})[int(r.get("n_gpus", 1))] = r       # the last line per N wins
    out = []
    for (impl, model, dtype), by_n in sorted(groups.items()):
        if len(by_n) < 2:
            continue
        ns = sorted(by_n)
        n0, v0 = ns[0], float(by_n[ns[0]]["value"])
        prev_n, prev_v = n0, v0
        for n in ns:
            v = float(by_n[n]["value"])
            gain = v / v0 if v0 > 0 else 0.0
            out.append({"impl": impl, "model": model, "dtype": dtype, "n_gpus": n,
                        "parallelism": (by_n[n].get("config") or {}).get("parallelism", "-"),
                        "value": v, "unit": by_n[n].get("unit", ""), "gain": gain,
                        "efficiency": gain / (n / n0),
                        "marginal_per_gpu": (v - prev_v) / (n - prev_n) if n > prev_n else 0.0})
            prev_n, prev_v = n, v
    return out


def capacity_efficiency(observed: float, stage_capacities) -> float:
    """Observed pipeline throughput over its ideal (the slowest stage's capacity); 0 when
    the ideal is undefined."""
    caps = [float(c) for c in stage_capacities]
    if not caps or min(caps) <= 0:
        return 0.0
    return observed / min(caps)


# ------------------------------------------------------------------------------------- rows
def _flat(d: dict, prefix: str = "") -> dict:
    out = {}
    for k, v in d.items():
        name = f"{prefix}{k}"
        if isinstance(v, dict):
            out.update(_flat(v, name + "."))
        elif isinstance(v, (list, tuple)):
            out[name] = json.dumps(v)
        else:
            out[name] = v
    return out


def rows_by_kind(records) -> dict[str, list[dict]]:
    """Flat table rows per kind (contracts, strategies and WAN evidence expand to one row per
    gate / candidate / profile)."""
    rows: dict[str, list[dict]] = {}
    for rec in records:
        k = kind(rec)
        if k == "contract":
            new = [{"contract": rec["contract"], "ok": rec.get("ok"), **_flat(r)} for r in rec["results"]]
        elif k == "strategy":
            new = [{"profile": rec.get("profile"), "selected": rec["selected"] == s.get("candidate"),
                    **_flat(s)} for s in rec["scores"]]
        elif k == "wan":
            new = [_flat(r) for r in rec["rows"]]
        elif k == "real_loopback":
            new = [{"checkpoint": rec.get("checkpoint"), "family": rec.get("family"),
                    "stages": len(rec.get("stages", [])), "tokens": len(rec["tokens"]),
                    "exact": rec.get("exact"), "reference": rec.get("reference"),
                    "seconds": rec.get("seconds")}]
        elif k == "other":
            new = [_flat(rec) if isinstance(rec, dict) else {"value": json.dumps(rec)}]
        else:
            new = [_flat(rec)]
        rows.setdefault(k, []).extend(new)
    return rows


def to_csv(rows: list[dict]) -> str:
    cols: list[str] = []
    for r in rows:
        cols += [c for c in r if c not in cols]
    buf = io.StringIO()
    w = csv.DictWriter(buf, fieldnames=cols, lineterminator="\n")
    w.writeheader()
    for r in rows:
        w.writerow(r)
    return buf.getvalue()


# --------------------------------------------------------------------------------- markdown
def to_markdown(records) -> str:
    out = []
    for rec in records:
        k = kind(rec)
        if k == "bench":
            cfg = rec.get("config", {})
            e2e = rec.get("e2e") or {}
            out += ["| impl | model | parallelism | GPUs | value | ms/step | TTFT ms | e2e | clocks |",
                    "|---|---|---|---|---|---|---|---|---|",
                    f"| {rec.get('impl', '-')} | {cfg.get('model', '-')} | {cfg.get('parallelism', '-')} | "
                    f"{rec.get('n_gpus')} | {rec['value']:.1f} {rec.get('unit', '')} | "
                    f"{rec.get('ms_per_step', 0):.3f} | {rec.get('ttft_ms_p50') or '-'} | "
                    f"{e2e.get('value', '-')} | {json.dumps(rec.get('clocks', {}))} |", ""]
        elif k == "contract":
            out += [f"contract `{rec['contract']}`: {'pass' if rec['ok'] else 'FAIL'}", "",
                    "| field | got | want | ok |", "|---|---|---|---|"]
            out += [f"| {r['field']} | {r.get('got')} | {r.get('op', '==')} {r.get('want')} | "
                    f"{r['ok']} |" for r in rec["results"]] + [""]
        elif k == "strategy":
            out += [f"profile `{rec['profile']}`: selected {rec['selected']}", "",
                    "| candidate | exact | ms / token | serial waits / token | bytes / token |",
                    "|---|---|---|---|---|"]
            out += [f"| {x['candidate']} | {x['feasible']} | {x['ms_per_token']:.2f} | "
                    f"{x['serial_waits_per_token']:.2f} | {x['payload_bytes_per_token']:.0f} |"
                    for x in rec["scores"]] + [""]
        elif k == "wan":
            from .wan_ring import markdown as wan_md
            out += [wan_md(rec["rows"]), ""]
        elif k == "loopback":
            from .loopback_matrix import markdown as lm_md
            out += [lm_md([rec]), ""]
        elif k == "expert_backend":
            from .expert_backends import markdown as eb_md
            out += [eb_md([rec]), ""]
        elif k == "real_loopback":
            stages = ", ".join(f"{s['worker']} {s['layers']}" for s in rec.get("stages", []))
            out += [f"real loopback `{rec.get('checkpoint')}` ({rec.get('family')}): "
                    f"{len(rec['tokens'])} tokens over [{stages}], exact={rec.get('exact')} "
                    f"against {rec.get('reference')}, {rec.get('seconds', 0):.1f} s", ""]
        else:
            out += ["```", json.dumps(rec, indent=1, default=str)[:2000], "```", ""]
    sc = scaling_rows(records)
    if sc:
        out += ["| impl | model | GPUs | parallelism | value | gain | efficiency | marginal / GPU |",
                "|---|---|---|---|---|---|---|---|"]
        out += [f"| {r['impl']} | {r['model']} | {r['n_gpus']} | {r['parallelism']} | "
                f"{r['value']:.1f} {r['unit']} | {r['gain']:.2f} | {r['efficiency']:.2f} | "
                f"{r['marginal_per_gpu']:.1f} |" for r in sc] + [""]
    return "\n".join(out)


# ------------------------------------------------------------------------------------- SVG
_PALETTE = ("#3b6ea5", "#d9822b", "#3a9a5b", "#b8433f", "#7d5ba6", "#8c6d46", "#c55f9b", "#6b6b6b")


def svg_bars(labels, values, title: str, unit: str = "", width: int = 640) -> str:
    """Horizontal bar chart, one bar per label."""
    labels = [str(l) for l in labels]
    values = [float(v) for v in values]
    if not values:
        return ""
    row, left, top = 22, 190, 28
    h = top + row * len(values) + 12
    vmax = max(max(values), 1e-12)
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{h}" '
             f'role="img" aria-label="{html.escape(title)}">',
             f'<text x="4" y="16" font-size="13" font-weight="bold">{html.escape(title)}</text>']
    span = width - left - 90
    for i, (lab, v) in enumerate(zip(labels, values)):
        y = top + i * row
        w = max(span * v / vmax, 0.0)
        parts += [f'<text x="{left - 6}" y="{y + 14}" font-size="11" text-anchor="end">'
                  f'{html.escape(lab[:32])}</text>',
                  f'<rect x="{left}" y="{y + 3}" width="{w:.1f}" height="{row - 6}" '
                  f'fill="{_PALETTE[i % len(_PALETTE)]}"/>',
                  f'<text x="{left + w + 4:.1f}" y="{y + 14}" font-size="11">'
                  f'{v:.4g} {html.escape(unit)}</text>']
    parts.append("</svg>")
    return "".join(parts)


def svg_lines(series: dict[str, list[tuple[float, float]]], title: str, xlabel: str, ylabel: str,
              width: int = 640, height: int = 300) -> str:
    """Line chart: ``series`` maps a name to (x, y) points; axes start at zero."""
    pts = [p for s in series.values() for p in s]
    if not pts:
        return ""
    left, right, top, bottom = 60, 150, 28, 40
    xmax = max(p[0] for p in pts) or 1.0
    ymax = max(p[1] for p in pts) or 1.0
    pw, ph = width - left - right, height - top - bottom

    def sx(x):
        return left + pw * x / xmax

    def sy(y):
        return top + ph * (1 - y / ymax)

    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" '
             f'role="img" aria-label="{html.escape(title)}">',
             f'<text x="4" y="16" font-size="13" font-weight="bold">{html.escape(title)}</text>',
             f'<line x1="{left}" y1="{top + ph}" x2="{left + pw}" y2="{top + ph}" stroke="#444"/>',
             f'<line x1="{left}" y1="{top}" x2="{left}" y2="{top + ph}" stroke="#444"/>',
             f'<text x="{left + pw / 2}" y="{height - 6}" font-size="11" text-anchor="middle">'
             f'{html.escape(xlabel)}</text>',
             f'<text x="12" y="{top + ph / 2}" font-size="11" text-anchor="middle" '
             f'transform="rotate(-90 12 {top + ph / 2})">{html.escape(ylabel)}</text>']
    for t in range(5):
        yv = ymax * t / 4
        parts.append(f'<text x="{left - 4}" y="{sy(yv) + 4:.1f}" font-size="10" '
                     f'text-anchor="end">{yv:.3g}</text>')
    for xv in sorted({p[0] for p in pts}):
        parts.append(f'<text x="{sx(xv):.1f}" y="{top + ph + 14}" font-size="10" '
                     f'text-anchor="middle">{xv:g}</text>')
    for i, (name, s) in enumerate(series.items()):
        c = _PALETTE[i % len(_PALETTE)]
        s = sorted(s)
        path = " ".join(f"{sx(x):.1f},{sy(y):.1f}" for x, y in s)
        parts.append(f'<polyline points="{path}" fill="none" stroke="{c}" stroke-width="2"/>')
        parts += [f'<circle cx="{sx(x):.1f}" cy="{sy(y):.1f}" r="3" fill="{c}"/>' for x, y in s]
        parts.append(f'<text x="{left + pw + 8}" y="{top + 14 + 16 * i}" font-size="11" '
                     f'fill="{c}">{html.escape(name[:24])}</text>')
    parts.append("</svg>")
    return "".join(parts)


def charts(records) -> list[str]:
    """The SVG charts the records support."""
    out = []
    bench = [r for r in records if kind(r) == "bench" and isinstance(r.get("value"), (int, float))]
    if bench:
        out.append(svg_bars([f"{r.get('impl', 'ours')} {(r.get('config') or {}).get('model', '')} "
                             f"x{r.get('n_gpus', 1)}" for r in bench],
                            [r["value"] for r in bench], "Bench throughput", bench[0].get("unit", "")))
    sc = scaling_rows(records)
    if sc:
        series: dict[str, list] = {}
        for r in sc:
            series.setdefault(f"{r['impl']} {r['model']}", []).append((r["n_gpus"], r["value"]))
        out.append(svg_lines(series, "Throughput against GPU count", "GPUs", sc[0]["unit"]))
        eff: dict[str, list] = {}
        for r in sc:
            eff.setdefault(f"{r['impl']} {r['model']}", []).append((r["n_gpus"], r["efficiency"]))
        out.append(svg_lines(eff, "Scaling efficiency (1.0 = linear)", "GPUs", "efficiency"))
    loop = [r for r in records if kind(r) == "loopback"]
    if loop:
        series = {}
        for r in loop:
            series.setdefault(f"{r['workers']} workers", []).append(
                (r["concurrency"], r["verified_tokens_per_s"]))
        out.append(svg_lines(series, "Verified tokens/s against concurrency", "concurrent requests",
                             "tokens/s"))
    wan = [row for r in records if kind(r) == "wan" for row in r["rows"]]
    if wan:
        out.append(svg_bars([r["profile"] for r in wan], [r["ms_per_token"] for r in wan],
                            "Stage-ring time per token by network profile", "ms"))
    eb = [r for r in records if kind(r) == "expert_backend"]
    if eb:
        out.append(svg_bars([r["backend"] for r in eb], [r["ms_per_forward"] for r in eb],
                            "Expert backends: time per forward", "ms"))
    return [c for c in out if c]


# ------------------------------------------------------------------------------------ HTML
def _html_table(rows: list[dict], limit: int = 200) -> str:
    cols: list[str] = []
    for r in rows:
        cols += [c for c in r if c not in cols]

    def cell(v):
        if isinstance(v, float):
            return f"{v:.4g}"
        if v is True or v is False:
            return f'<span class="{"ok" if v else "bad"}">{v}</span>'
        return html.escape(str(v))

    head = "".join(f"<th>{html.escape(c)}</th>" for c in cols)
    body = "".join("<tr>" + "".join(f"<td>{cell(r.get(c, ''))}</td>" for c in cols) + "</tr>"
                   for r in rows[:limit])
    if len(rows) > limit:
        body += f'<tr><td colspan="{len(cols)}">{len(rows) - limit} more rows in the CSV</td></tr>'
    return f"<table><thead><tr>{head}</tr></thead><tbody>{body}</tbody></table>"


def summary(records) -> dict:
    rows = rows_by_kind(records)
    contracts = [r for r in records if kind(r) == "contract"]
    exact = [r.get("exact") for r in records if kind(r) in ("real_loopback", "expert_backend")]
    exact += [row.get("exact_tokens") for r in records if kind(r) == "wan" for row in r["rows"]]
    failed = [r["contract"] for r in contracts if not r.get("ok")] + \
        (["exactness"] if any(e is False for e in exact) else [])
    return {"records": len(records), "kinds": {k: len(v) for k, v in rows.items()},
            "contracts_passed": sum(1 for r in contracts if r.get("ok")),
            "contracts_failed": sum(1 for r in contracts if not r.get("ok")),
            "exactness_checks": len(exact), "status": "FAIL" if failed else "PASS",
            "failed": failed, "scaling": scaling_rows(records)}


def to_html(records, title: str = "Evidence report") -> str:
    s = summary(records)
    rows = rows_by_kind(records)
    parts = ["<!doctype html><html><head><meta charset='utf-8'>",
             f"<title>{html.escape(title)}</title><style>",
             "body{font-family:sans-serif;margin:24px;max-width:1100px}"
             "table{border-collapse:collapse;margin:8px 0 20px;font-size:12px}"
             "td,th{border:1px solid #ccc;padding:3px 6px;text-align:left}"
             "th{background:#f0f0f0}.ok{color:#2a7a3a}.bad{color:#b00;font-weight:bold}"
             "figure{margin:10px 0}",
             "</style></head><body>",
             f"<h1>{html.escape(title)}</h1>",
             f"<p>Status: <span class='{'ok' if s['status'] == 'PASS' else 'bad'}'>{s['status']}</span>"
             f" &middot; {s['records']} records &middot; contracts passed {s['contracts_passed']}, "
             f"failed {s['contracts_failed']} &middot; exactness checks {s['exactness_checks']}</p>"]
    if s["failed"]:
        parts.append("<p class='bad'>Failed: " + html.escape(", ".join(s["failed"])) + "</p>")
    for c in charts(records):
        parts.append(f"<figure>{c}</figure>")
    if s["scaling"]:
        parts += ["<h2>Scaling</h2>", _html_table(s["scaling"])]
    for k in KINDS:
        if k in rows:
            parts += [f"<h2>{html.escape(k)}</h2>", _html_table(rows[k])]
    parts.append("</body></html>")
    return "\n".join(parts)


def write_bundle(records, out_dir, title: str = "Evidence report") -> dict:
    """``report.html``, ``report.md``, ``summary.json``, ``records.jsonl`` and one CSV per
    record kind under OUT_DIR; returns the summary."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    (out / "report.html").write_text(to_html(records, title))
    (out / "report.md").write_text(to_markdown(records))
    (out / "records.jsonl").write_text("".join(json.dumps(r, default=str) + "\n" for r in records))
    for k, rows in rows_by_kind(records).items():
        (out / f"{k}.csv").write_text(to_csv(rows))
    s = summary(records)
    sc = s["scaling"]
    if sc:
        (out / "scaling.csv").write_text(to_csv(sc))
    (out / "summary.json").write_text(json.dumps(s, indent=1, default=str))
    return s
