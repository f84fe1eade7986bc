"""Timeline viewer for event logs (C34).

Renders the JSONL written by :class:`psrl_b200.utils.events.EventLog` (begin /
end spans per actor and event type) into a self-contained HTML page with one
lane per actor and one colour per event type — the role of the reference's
Flask log visualiser, without a server.

    python -m psrl_b200.utils.visualize events.jsonl timeline.html
"""

from __future__ import annotations

import html
import json
import sys

COLORS = {"PULL": "#4e79a7", "PUSH": "#f28e2b", "BUFFER_READY": "#59a14f", "INIT": "#bab0ac", "TRAIN": "#e15759",
          "GEN": "#76b7b2", "VAL": "#edc948", "WAIT": "#9c755f", "SWITCH": "#b07aa1", "OTHER": "#aaaaaa"}


def spans(events: list[dict]) -> list[dict]:
    open_: dict = {}
    out = []
    for e in sorted(events, key=lambda x: x["ts"]):
        key = (e.get("actor"), e.get("name"), e.get("type"))
        if e.get("phase") == "begin":
            open_[key] = e
        elif e.get("phase") == "end" and key in open_:
            b = open_.pop(key)
            out.append({"actor": e.get("actor"), "name": e.get("name"), "type": e.get("type"),
                        "start": b["ts"], "end": e["ts"]})
    return out


def render(events: list[dict], title: str = "psrl_b200 timeline") -> str:
    sp = spans(events)
    if not sp:
        return f"<html><body><h3>{html.escape(title)}</h3><p>no spans</p></body></html>"
    t0 = min(s["start"] for s in sp)
    t1 = max(s["end"] for s in sp)
    width = 1200.0
    scale = width / max(1e-9, t1 - t0)
    actors = sorted({s["actor"] for s in sp})
    rows = []
    for i, a in enumerate(actors):
        y = 30 + i * 28
        rows.append(f'<text x="0" y="{y + 14}" font-size="11">{html.escape(str(a))}</text>')
        for s in (x for x in sp if x["actor"] == a):
            x = 120 + (s["start"] - t0) * scale
            w = max(1.0, (s["end"] - s["start"]) * scale)
            c = COLORS.get(s["type"], "#999")
            tip = html.escape(f'{s["name"]} {s["end"] - s["start"]:.3f}s')
            rows.append(f'<rect x="{x:.1f}" y="{y}" width="{w:.1f}" height="20" fill="{c}"><title>{tip}</title></rect>')
    legend = " ".join(f'<span style="background:{c};padding:2px 6px;margin:2px">{k}</span>' for k, c in COLORS.items())
    h = 40 + 28 * len(actors)
    return (f"<html><head><title>{html.escape(title)}</title></head><body><h3>{html.escape(title)}</h3>"
            f"<div>{legend}</div><svg width='{width + 140}' height='{h}'>{''.join(rows)}</svg>"
            f"<p>span {t1 - t0:.2f}s</p></body></html>")


def main(argv=None) -> int:
    """``visualize SRC... OUT.html``: SRC is an events file (JSON lines) or a
    directory of them (one per rank, as ``trainer.event_log_dir`` writes); all
    ranks' spans go on one timeline."""
    import os
    argv = argv if argv is not None else sys.argv[1:]
    *srcs, dst = argv
    files = []
    for src in srcs:
        if os.path.isdir(src):
            files += sorted(os.path.join(src, f) for f in os.listdir(src) if f.endswith(".jsonl"))
        else:
            files.append(src)
    events = []
    for f in files:
        with open(f) as fh:
            events += [json.loads(ln) for ln in fh if ln.strip()]
    with open(dst, "w") as fh:
        fh.write(render(events))
    return 0


if __name__ == "__main__":
    sys.exit(main())
