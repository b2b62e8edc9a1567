"""Accounts, JWT roles (RBAC) and CORS on the HTTP API (CPU, tiny model)."""
import os
import time

import pytest
from fastapi.testclient import TestClient

from vramancer_b200.serving.auth import Auth, AuthError, CorsPolicy, jwt_decode, jwt_encode, required_role


def test_jwt_roundtrip_tamper_and_expiry():
    tok = jwt_encode({"sub": "a", "role": "ops", "exp": time.time() + 60}, "k1")
    assert jwt_decode(tok, "k1")["role"] == "ops"
    with pytest.raises(AuthError):
        jwt_decode(tok, "k2")
    head, body, sig = tok.split(".")
    forged = jwt_encode({"sub": "a", "role": "admin", "exp": time.time() + 60}, "k1").split(".")[1]
    with pytest.raises(AuthError):
        jwt_decode(f"{head}.{forged}.{sig}", "k1")
    old = jwt_encode({"sub": "a", "exp": time.time() - 1}, "k1")
    with pytest.raises(AuthError, match="expired"):
        jwt_decode(old, "k1")


def test_users_passwords_and_refresh_rotation(tmp_path):
    f = str(tmp_path / "users.json")
    a = Auth(secret="s", users_file=f)
    a.create_user("alice", "pw1", "ops")
    with pytest.raises(AuthError):
        a.create_user("alice", "x")
    assert a.verify("alice", "pw1") and not a.verify("alice", "bad") and not a.verify("bob", "pw1")
    t = a.login("alice", "pw1")
    assert a.access_claims(t["access"])["role"] == "ops"
    assert a.access_claims(t["refresh"]) is None            # a refresh token is not an access token
    t2 = a.refresh(t["refresh"])
    with pytest.raises(AuthError):
        a.refresh(t["refresh"])                              # single use
    assert a.access_claims(t2["access"])["sub"] == "alice"
    assert a.change_password("alice", "pw1", "pw2") and a.verify("alice", "pw2")
    b = Auth(secret="s", users_file=f)                       # persisted, hashes only
    assert b.verify("alice", "pw2") and "pw2" not in open(f).read()


def test_cors_policy():
    c = CorsPolicy("http://a.example,http://b.example")
    assert c.allowed(None) and c.allowed("http://a.example") and not c.allowed("http://evil.example")
    assert c.headers("http://a.example")["Access-Control-Allow-Origin"] == "http://a.example"
    assert CorsPolicy("*").allowed("http://anything")
    assert required_role("POST", "/api/models/load") == "ops" and required_role("GET", "/v1/models") is None


@pytest.fixture(scope="module")
def app_client():
    from vramancer_b200.pipeline import InferencePipeline
    from vramancer_b200.serving.api import create_app
    saved = {k: os.environ.get(k) for k in ("VRM_API_TOKEN", "VRM_AUTH_SECRET", "VRM_DISABLE_RATE_LIMIT",
                                            "VRM_CORS_ORIGINS", "VRM_DEFAULT_ADMIN_PASS")}
    os.environ.update({"VRM_API_TOKEN": "static", "VRM_AUTH_SECRET": "jwtsecret", "VRM_DISABLE_RATE_LIMIT": "1",
                       "VRM_CORS_ORIGINS": "http://ok.example", "VRM_DEFAULT_ADMIN_PASS": "rootpw"})
    pipe = InferencePipeline().load("tiny-qwen2", device="cpu", max_model_len=128, max_batch=2)
    app = create_app(pipe)
    with TestClient(app) as c:
        yield c, app
    pipe.shutdown()
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


def test_login_roles_and_rbac(app_client):
    c, app = app_client
    r = c.post("/api/auth/login", json={"username": "admin", "password": "wrong"})
    assert r.status_code == 401
    adm = c.post("/api/auth/login", json={"username": "admin", "password": "rootpw"}).json()
    H = lambda t: {"Authorization": f"Bearer {t}"}
    r = c.post("/api/auth/users", json={"username": "u1", "password": "p1", "role": "user"}, headers=H(adm["access"]))
    assert r.status_code == 200, r.text
    c.post("/api/auth/users", json={"username": "o1", "password": "p2", "role": "ops"}, headers=H(adm["access"]))
    user = c.post("/api/auth/login", json={"username": "u1", "password": "p1"}).json()
    ops = c.post("/api/auth/login", json={"username": "o1", "password": "p2"}).json()
    assert c.get("/api/auth/me", headers=H(user["access"])).json() == {"user": "u1", "role": "user"}
    # inference is open to every role; user management and model loading are not
    assert c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 2}, headers=H(user["access"])).status_code == 200
    assert c.get("/api/auth/users", headers=H(user["access"])).status_code == 403
    assert c.get("/api/nodes", headers=H(user["access"])).status_code == 403
    assert c.get("/api/nodes", headers=H(ops["access"])).status_code == 200
    assert c.get("/api/auth/users", headers=H(ops["access"])).status_code == 403
    assert c.get("/api/auth/users", headers=H("static")).status_code == 200     # static token = admin
    assert c.get("/v1/models", headers=H("garbage")).status_code == 401
    # refresh rotation over HTTP
    r2 = c.post("/api/auth/refresh", json={"refresh": user["refresh"]})
    assert r2.status_code == 200 and c.post("/api/auth/refresh", json={"refresh": user["refresh"]}).status_code == 401


def test_cors_on_the_api(app_client):
    c, _ = app_client
    H = {"Authorization": "Bearer static"}
    assert c.get("/v1/models", headers={**H, "Origin": "http://evil.example"}).status_code == 403
    r = c.get("/v1/models", headers={**H, "Origin": "http://ok.example"})
    assert r.status_code == 200 and r.headers["access-control-allow-origin"] == "http://ok.example"
    pre = c.options("/v1/completions", headers={"Origin": "http://ok.example",
                                                "Access-Control-Request-Method": "POST"})
    assert pre.status_code == 204 and "POST" in pre.headers["access-control-allow-methods"]
