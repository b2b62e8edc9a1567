"""Reference arm of bench.py: runs the unmodified reference (installed into
baseline/_ref) through its own public API on the same metric and config."""
import json


def run(args, metric):
    print(json.dumps({"impl": "reference", "unavailable": "reference arm not wired yet"}), flush=True)
