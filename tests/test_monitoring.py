"""Monitoring provisioning: the alert rules and the Grafana dashboard parse and refer
only to metrics that vramancer_b200 exports; the files copy out."""
import json
import re

import pytest
import yaml

from vramancer_b200.utils import monitoring
from vramancer_b200.utils.observability import Metrics


def _exported():
    prom = pytest.importorskip("prometheus_client")
    m = Metrics(registry=prom.CollectorRegistry())
    names = set()
    for fam in m.registry.collect():
        names.add(fam.name)
        for s in fam.samples:
            names.add(s.name)
    return names


def _metric_names(expr):
    return set(re.findall(r"\bvrm_[a-z_]+\b", expr))


def _known(n, names):
    """A sample name of an exported family (counters add _total, histograms _bucket /
    _sum / _count; labelled families have no samples until a label is set)."""
    base = re.sub(r"_(bucket|sum|count)$", "", n)
    return any(x in names for x in (n, base, re.sub(r"_total$", "", base)))


def test_alert_rules_use_exported_metrics():
    names = _exported()
    rules = yaml.safe_load(open(monitoring.path("alerting_rules.yml")))
    count = 0
    for g in rules["groups"]:
        for r in g["rules"]:
            count += 1
            assert r["alert"] and r["expr"] and r["labels"]["severity"] in ("info", "warning", "critical")
            for n in _metric_names(r["expr"]):
                assert _known(n, names), (r["alert"], n)
    assert count >= 20


def test_dashboard_and_scrape_config(tmp_path):
    names = _exported()
    dash = json.load(open(monitoring.path("grafana_dashboard.json")))
    assert dash["panels"]
    for p in dash["panels"]:
        for t in p["targets"]:
            for n in _metric_names(t["expr"]):
                assert _known(n, names), (p["title"], n)
    cfg = yaml.safe_load(open(monitoring.path("prometheus.yml")))
    assert cfg["rule_files"] == ["alerting_rules.yml"]
    assert any("9108" in t for j in cfg["scrape_configs"] for s in j["static_configs"] for t in s["targets"])
    out = monitoring.write(str(tmp_path / "mon"))
    assert len(out) == 3 and all(open(p).read() for p in out)
