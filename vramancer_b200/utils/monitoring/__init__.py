"""Monitoring provisioning for a deployment: Prometheus scrape configuration
(prometheus.yml), alert rules over the exported metrics (alerting_rules.yml) and a
Grafana dashboard (grafana_dashboard.json).

    python -m vramancer_b200.utils.monitoring /etc/vramancer/monitoring

copies the three files into a directory for Prometheus / Grafana to load.

Reference parity: monitoring/alerting_rules.yml, monitoring/prometheus.yml (the
reference's Prometheus / Grafana / Alertmanager provisioning).
"""
from __future__ import annotations

import os
import shutil
import sys
from typing import List

FILES = ("prometheus.yml", "alerting_rules.yml", "grafana_dashboard.json")
HERE = os.path.dirname(os.path.abspath(__file__))


def path(name: str) -> str:
    if name not in FILES:
        raise KeyError(name)
    return os.path.join(HERE, name)


def write(dest: str) -> List[str]:
    """Copies the provisioning files into `dest` (created if needed); returns the paths."""
    os.makedirs(dest, exist_ok=True)
    out = []
    for f in FILES:
        shutil.copyfile(path(f), os.path.join(dest, f))
        out.append(os.path.join(dest, f))
    return out


if __name__ == "__main__":
    for p in write(sys.argv[1] if len(sys.argv) > 1 else "."):
        print(p)
