"""Credit ledger for shared serving: per-user API keys and a VRAM-credit balance.

Keys have the form `sk-VRAM-<random>`; only their SHA-256 is stored.  A completion
request made with such a key is refused with 401 when the key is unknown and with 402
when the balance is exhausted; an admitted request is charged for the tokens it may
generate (max_tokens) at CREDIT_PER_TOKEN.  Nodes registered to a user earn
CREDIT_PER_BLOCK per block they compute for others.  The ledger is one SQLite file
(VRM_LEDGER_DB); every method takes the lock and its own connection, so it is safe from
the API's worker threads.

Reference parity: core/production_api.py:597-655 (sk-VRAM- key check, 401 / 402, credit
consumption of max_tokens), _deprecated/swarm_ledger.py:25-160 (users with hashed keys,
100 initial credits, 0.001 credit per token, 0.0005 per block for a user's node).
"""
from __future__ import annotations

import contextlib
import hashlib
import secrets
import sqlite3
import threading
import uuid
from typing import Any, Dict, Iterator, Optional, Tuple

KEY_PREFIX = "sk-VRAM-"
INITIAL_CREDITS = 100.0
CREDIT_PER_TOKEN = 0.001
CREDIT_PER_BLOCK = 0.0005


def _hash(key: str) -> str:
    return hashlib.sha256(key.encode()).hexdigest()


class CreditLedger:
    def __init__(self, path: str):
        self.path = path
        self._lock = threading.Lock()
        with self._tx() as c:
            c.execute("CREATE TABLE IF NOT EXISTS users (id TEXT PRIMARY KEY, key_hash TEXT UNIQUE, alias TEXT, "
                      "credits REAL NOT NULL, created REAL DEFAULT (julianday('now')))")
            c.execute("CREATE TABLE IF NOT EXISTS nodes (node_id TEXT PRIMARY KEY, user_id TEXT NOT NULL)")

    @contextlib.contextmanager
    def _tx(self) -> Iterator[sqlite3.Connection]:
        """One locked transaction on a fresh connection (committed, then closed)."""
        with self._lock:
            c = sqlite3.connect(self.path, timeout=10.0)
            try:
                with c:
                    yield c
            finally:
                c.close()

    # ------------------------------------------------------------------ users
    def create_user(self, alias: str, credits: float = INITIAL_CREDITS) -> Tuple[str, str]:
        """(user id, API key); the key is returned once and stored only as a hash."""
        uid = str(uuid.uuid4())
        key = KEY_PREFIX + secrets.token_urlsafe(32)
        with self._tx() as c:
            c.execute("INSERT INTO users (id, key_hash, alias, credits) VALUES (?, ?, ?, ?)",
                      (uid, _hash(key), alias, float(credits)))
        return uid, key

    def verify(self, api_key: str) -> Optional[Dict[str, Any]]:
        """{"id", "alias", "credits"} of the key's user, or None."""
        if not api_key.startswith(KEY_PREFIX):
            return None
        with self._tx() as c:
            row = c.execute("SELECT id, alias, credits FROM users WHERE key_hash = ?", (_hash(api_key),)).fetchone()
        return {"id": row[0], "alias": row[1], "credits": row[2]} if row else None

    def balance(self, user_id: str) -> Optional[float]:
        with self._tx() as c:
            row = c.execute("SELECT credits FROM users WHERE id = ?", (user_id,)).fetchone()
        return None if row is None else float(row[0])

    def consume(self, user_id: str, tokens: int) -> bool:
        """Charges `tokens` x CREDIT_PER_TOKEN; False (nothing charged) when the balance is
        short or the user unknown.  Check and debit are one statement."""
        cost = max(0, int(tokens)) * CREDIT_PER_TOKEN
        with self._tx() as c:
            cur = c.execute("UPDATE users SET credits = credits - ? WHERE id = ? AND credits >= ?",
                            (cost, user_id, cost))
            return cur.rowcount == 1

    def add_credits(self, user_id: str, amount: float) -> bool:
        with self._tx() as c:
            return c.execute("UPDATE users SET credits = credits + ? WHERE id = ?",
                             (float(amount), user_id)).rowcount == 1

    # ------------------------------------------------------------------ nodes
    def register_node(self, node_id: str, user_id: str) -> None:
        with self._tx() as c:
            c.execute("INSERT OR REPLACE INTO nodes (node_id, user_id) VALUES (?, ?)", (node_id, user_id))

    def reward_node(self, node_id: str, blocks: int) -> bool:
        """Credits the node's owner CREDIT_PER_BLOCK per block computed for others."""
        with self._tx() as c:
            row = c.execute("SELECT user_id FROM nodes WHERE node_id = ?", (node_id,)).fetchone()
            if row is None:
                return False
            c.execute("UPDATE users SET credits = credits + ? WHERE id = ?",
                      (max(0, int(blocks)) * CREDIT_PER_BLOCK, row[0]))
            return True
