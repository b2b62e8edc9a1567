"""SQLite persistence of multi-step workflows (id, name, status, params, result, times).

Reference parity: core/persistence.py (SQLite workflow store).
"""
from __future__ import annotations

import json
import sqlite3
import threading
import time
import uuid
from typing import Any, Dict, List, Optional


class WorkflowStore:
    def __init__(self, path: str = "vramancer_workflows.sqlite"):
        self._db = sqlite3.connect(path, check_same_thread=False)
        self._lock = threading.Lock()
        with self._lock:
            self._db.execute("CREATE TABLE IF NOT EXISTS workflows (id TEXT PRIMARY KEY, name TEXT, status TEXT, "
                             "params TEXT, result TEXT, created REAL, updated REAL)")
            self._db.commit()

    def create(self, name: str, params: Optional[Dict[str, Any]] = None) -> str:
        wid = uuid.uuid4().hex
        now = time.time()
        with self._lock:
            self._db.execute("INSERT INTO workflows VALUES (?, ?, ?, ?, ?, ?, ?)",
                             (wid, name, "pending", json.dumps(params or {}), None, now, now))
            self._db.commit()
        return wid

    def update(self, wid: str, status: Optional[str] = None, result: Any = None) -> None:
        with self._lock:
            if status is not None:
                self._db.execute("UPDATE workflows SET status = ?, updated = ? WHERE id = ?", (status, time.time(), wid))
            if result is not None:
                self._db.execute("UPDATE workflows SET result = ?, updated = ? WHERE id = ?",
                                 (json.dumps(result), time.time(), wid))
            self._db.commit()

    def _row(self, r) -> Dict[str, Any]:
        return {"id": r[0], "name": r[1], "status": r[2], "params": json.loads(r[3] or "{}"),
                "result": json.loads(r[4]) if r[4] else None, "created": r[5], "updated": r[6]}

    def get(self, wid: str) -> Optional[Dict[str, Any]]:
        with self._lock:
            r = self._db.execute("SELECT * FROM workflows WHERE id = ?", (wid,)).fetchone()
        return self._row(r) if r else None

    def list(self, status: Optional[str] = None) -> List[Dict[str, Any]]:
        q = "SELECT * FROM workflows" + (" WHERE status = ?" if status else "") + " ORDER BY created"
        with self._lock:
            rows = self._db.execute(q, (status,) if status else ()).fetchall()
        return [self._row(r) for r in rows]

    def close(self) -> None:
        self._db.close()
