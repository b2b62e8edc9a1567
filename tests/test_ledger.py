"""Credit ledger: sk-VRAM- keys, 401 for unknown keys, 402 for spent balances, the
charge of max_tokens, node rewards, and the same through the HTTP API on a CPU model."""
import os
import threading

import pytest
from fastapi.testclient import TestClient

from vramancer_b200.serving.ledger import CREDIT_PER_BLOCK, CREDIT_PER_TOKEN, INITIAL_CREDITS, CreditLedger


def test_ledger_keys_balances_and_rewards(tmp_path):
    lg = CreditLedger(str(tmp_path / "l.db"))
    uid, key = lg.create_user("alice")
    assert key.startswith("sk-VRAM-") and lg.verify(key)["id"] == uid
    assert lg.verify("sk-VRAM-nope") is None and lg.verify("other") is None
    assert lg.balance(uid) == INITIAL_CREDITS
    assert lg.consume(uid, 1000) and lg.balance(uid) == pytest.approx(INITIAL_CREDITS - 1000 * CREDIT_PER_TOKEN)
    assert not lg.consume(uid, 10 ** 9)                       # short: nothing charged
    assert lg.balance(uid) == pytest.approx(INITIAL_CREDITS - 1.0)
    lg.register_node("node-1", uid)
    assert lg.reward_node("node-1", 2000) and not lg.reward_node("node-x", 1)
    assert lg.balance(uid) == pytest.approx(INITIAL_CREDITS - 1.0 + 2000 * CREDIT_PER_BLOCK)
    with open(tmp_path / "l.db", "rb") as f:
        assert key.encode() not in f.read()                   # only the hash is stored


def test_ledger_concurrent_charges_are_exact(tmp_path):
    lg = CreditLedger(str(tmp_path / "c.db"))
    uid, _ = lg.create_user("bob", credits=10.0)

    def worker():
        for _ in range(50):
            lg.consume(uid, 100)                              # 0.1 credit each
    ts = [threading.Thread(target=worker) for _ in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert lg.balance(uid) == pytest.approx(0.0, abs=1e-9)   # 100 charges fit, the rest refused


@pytest.fixture(scope="module")
def ledger_client(tmp_path_factory):
    from vramancer_b200.pipeline import InferencePipeline
    from vramancer_b200.serving.api import create_app
    db = tmp_path_factory.mktemp("ledger") / "api.db"
    old = {k: os.environ.get(k) for k in ("VRM_API_TOKEN", "VRM_DISABLE_RATE_LIMIT", "VRM_LEDGER_DB")}
    os.environ.update({"VRM_API_TOKEN": "admintoken", "VRM_DISABLE_RATE_LIMIT": "1", "VRM_LEDGER_DB": str(db)})
    pipe = InferencePipeline(enable_metrics=False).load("tiny-qwen2", device="cpu", max_model_len=256, max_batch=4)
    try:
        with TestClient(create_app(pipe)) as c:
            yield c
    finally:
        pipe.shutdown()
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def test_api_ledger_flow(ledger_client):
    c = ledger_client
    admin = {"Authorization": "Bearer admintoken"}
    r = c.post("/api/ledger/users", json={"alias": "carol", "credits": 1.0}, headers=admin)
    assert r.status_code == 200
    key, uid = r.json()["api_key"], r.json()["id"]
    user = {"Authorization": f"Bearer {key}"}
    # a ledger user may not create users
    assert c.post("/api/ledger/users", json={"alias": "x"}, headers=user).status_code == 403
    assert c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 4},
                  headers={"Authorization": "Bearer sk-VRAM-unknown"}).status_code == 401
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 100},
               headers=user)
    assert r.status_code == 200, r.text
    bal = c.get("/api/ledger/balance", headers=user).json()["credit_balance"]
    assert bal == pytest.approx(1.0 - 100 * CREDIT_PER_TOKEN)
    c.app.state.ledger.add_credits(uid, -bal)                  # spend the rest
    r = c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 4}, headers=user)
    assert r.status_code == 402 and r.json()["credit_balance"] <= 0
