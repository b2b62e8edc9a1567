"""Accounts, JWT access / refresh tokens, role-based access control and CORS.

  users     PBKDF2-HMAC-SHA256 password hashes (per-user random salt), in memory, or
            persisted as JSON when VRM_AUTH_USERS_FILE is set; roles user < ops < admin
  tokens    HS256 JWTs (RFC 7519, written here with hmac / base64: no extra package)
            signed with VRM_AUTH_SECRET; access tokens carry sub / role / exp / typ,
            refresh tokens are single-use (rotated on every refresh)
  RBAC      ROLE_REQUIRED maps a route (and method) to the lowest role that may call
            it; a request's role comes from its JWT, the static VRM_API_TOKEN counts as
            admin, and with no credentials configured at all (development) everyone is
            admin, so the map stays consistent
  CORS      VRM_CORS_ORIGINS (comma-separated, "*" for any; default the localhost
            origins): a request whose Origin is not allowed gets 403, allowed origins
            get the Access-Control-Allow-* headers and preflights are answered

Reference parity: core/auth_strong.py:24-164 (users, pbkdf2 120k rounds, HS256
access / refresh with rotation, roles user / ops / admin, default admin bootstrap),
core/security/__init__.py:241-318 (CORS origin check, role from JWT or shared secret,
RBAC ladder).  Same environment names (VRM_AUTH_SECRET, VRM_AUTH_EXP,
VRM_AUTH_REFRESH_EXP, VRM_CORS_ORIGINS, VRM_DEFAULT_ADMIN_PASS) so deployments keep
their configuration.
"""
from __future__ import annotations

import base64
import hashlib
import hmac
import json
import os
import secrets
import threading
import time
from dataclasses import asdict, dataclass
from typing import Dict, Optional, Tuple

ROLES = {"user": 0, "ops": 1, "admin": 2}
PBKDF2_ROUNDS = 120_000

# (method or "*", path) -> lowest role allowed.  Inference routes need "user".
ROLE_REQUIRED: Dict[Tuple[str, str], str] = {
    ("POST", "/api/models/load"): "ops",
    ("POST", "/api/ledger/users"): "admin",
    ("POST", "/api/lora"): "ops",
    ("*", "/api/nodes"): "ops",
    ("POST", "/api/worker/load_partial"): "ops",
    ("POST", "/api/benchmark"): "ops",
    ("POST", "/api/swarm/awaken"): "admin",
    ("*", "/api/auth/users"): "admin",
    ("*", "/api/audit"): "admin",
}


class AuthError(ValueError):
    pass


# --------------------------------------------------------------------------- JWT (HS256)
def _b64(b: bytes) -> str:
    return base64.urlsafe_b64encode(b).rstrip(b"=").decode()


def _unb64(s: str) -> bytes:
    return base64.urlsafe_b64decode(s + "=" * (-len(s) % 4))


def jwt_encode(payload: dict, secret: str) -> str:
    head = _b64(json.dumps({"alg": "HS256", "typ": "JWT"}, separators=(",", ":")).encode())
    body = _b64(json.dumps(payload, separators=(",", ":"), sort_keys=True).encode())
    sig = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
    return f"{head}.{body}.{_b64(sig)}"


def jwt_decode(token: str, secret: str, now: Optional[float] = None) -> dict:
    """Payload of a valid, unexpired HS256 token; AuthError otherwise."""
    try:
        head, body, sig = token.split(".")
        h = json.loads(_unb64(head))
    except Exception:
        raise AuthError("malformed token")
    if h.get("alg") != "HS256":
        raise AuthError("unsupported token algorithm")
    want = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
    try:
        got = _unb64(sig)
    except Exception:
        raise AuthError("malformed token")
    if not hmac.compare_digest(want, got):
        raise AuthError("bad token signature")
    p = json.loads(_unb64(body))
    if float(p.get("exp", 0)) < (time.time() if now is None else now):
        raise AuthError("token expired")
    return p


# --------------------------------------------------------------------------- users
@dataclass
class User:
    username: str
    pwd_hash: str
    salt: str
    role: str = "user"
    must_change_password: bool = False


def _hash(password: str, salt: str) -> str:
    return hashlib.pbkdf2_hmac("sha256", password.encode(), salt.encode(), PBKDF2_ROUNDS).hex()


class Auth:
    """User store + token service of one API server."""

    def __init__(self, secret: Optional[str] = None, users_file: Optional[str] = None):
        self._secret = secret or os.environ.get("VRM_AUTH_SECRET") or ""
        self._volatile = not self._secret
        if not self._secret:
            # development: tokens die with the process
            self._secret = secrets.token_hex(32)
        self.users_file = users_file or os.environ.get("VRM_AUTH_USERS_FILE") or None
        self.users: Dict[str, User] = {}
        self._refresh: Dict[str, Tuple[str, float]] = {}
        self._lock = threading.Lock()
        if self.users_file and os.path.exists(self.users_file):
            with open(self.users_file) as f:
                for d in json.load(f):
                    self.users[d["username"]] = User(**d)

    @property
    def configured(self) -> bool:
        """True when tokens survive a restart (VRM_AUTH_SECRET set) or accounts exist."""
        return not self._volatile or bool(self.users)

    # ----------------------------------------------------------------- accounts
    def _save(self) -> None:
        if not self.users_file:
            return
        tmp = self.users_file + ".tmp"
        fd = os.open(tmp, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        with os.fdopen(fd, "w") as f:
            json.dump([asdict(u) for u in self.users.values()], f)
        os.replace(tmp, self.users_file)

    def create_user(self, username: str, password: str, role: str = "user",
                    must_change_password: bool = False) -> User:
        if role not in ROLES:
            raise AuthError(f"unknown role {role!r}")
        if not username or not password:
            raise AuthError("username and password required")
        with self._lock:
            if username in self.users:
                raise AuthError("user exists")
            salt = secrets.token_hex(16)
            u = User(username, _hash(password, salt), salt, role, must_change_password)
            self.users[username] = u
            self._save()
        return u

    def delete_user(self, username: str) -> bool:
        with self._lock:
            ok = self.users.pop(username, None) is not None
            self._save()
        return ok

    def verify(self, username: str, password: str) -> bool:
        u = self.users.get(username)
        if u is None:
            _hash(password, "x" * 32)        # same work whether or not the user exists
            return False
        return hmac.compare_digest(_hash(password, u.salt), u.pwd_hash)

    def change_password(self, username: str, old: str, new: str) -> bool:
        if not new or not self.verify(username, old):
            return False
        with self._lock:
            u = self.users[username]
            u.salt = secrets.token_hex(16)
            u.pwd_hash = _hash(new, u.salt)
            u.must_change_password = False
            self._save()
        return True

    def ensure_default_admin(self, production: bool = False) -> Optional[str]:
        """Creates "admin" when there is no account: with VRM_DEFAULT_ADMIN_PASS, else a
        random password that must be changed (returned, never logged).  Not in
        production, where accounts must be created explicitly."""
        if self.users or production:
            return None
        pw = os.environ.get("VRM_DEFAULT_ADMIN_PASS")
        force = pw is None
        pw = pw or secrets.token_urlsafe(16)
        self.create_user("admin", pw, "admin", must_change_password=force)
        return pw

    # ----------------------------------------------------------------- tokens
    def issue(self, username: str, now: Optional[float] = None) -> dict:
        u = self.users[username]
        t = int(time.time() if now is None else now)
        exp_a = t + int(os.environ.get("VRM_AUTH_EXP", "900"))
        exp_r = t + int(os.environ.get("VRM_AUTH_REFRESH_EXP", "86400"))
        access = jwt_encode({"sub": username, "role": u.role, "iat": t, "exp": exp_a, "typ": "access",
                             "pwd_change": u.must_change_password}, self._secret)
        refresh = jwt_encode({"sub": username, "iat": t, "exp": exp_r, "typ": "refresh",
                              "jti": secrets.token_hex(8)}, self._secret)
        with self._lock:
            self._refresh[refresh] = (username, float(exp_r))
        return {"access": access, "refresh": refresh, "token_type": "bearer", "expires_in": exp_a - t,
                "role": u.role}

    def login(self, username: str, password: str) -> dict:
        if not self.verify(username, password):
            raise AuthError("invalid credentials")
        return self.issue(username)

    def refresh(self, token: str) -> dict:
        p = jwt_decode(token, self._secret)
        if p.get("typ") != "refresh":
            raise AuthError("not a refresh token")
        with self._lock:
            rec = self._refresh.pop(token, None)        # single use: rotated
        if rec is None or rec[1] < time.time() or rec[0] not in self.users:
            raise AuthError("refresh token revoked or expired")
        return self.issue(rec[0])

    def access_claims(self, token: str) -> Optional[dict]:
        """Claims of a valid access token, else None."""
        try:
            p = jwt_decode(token, self._secret)
        except (AuthError, ValueError):
            return None
        if p.get("typ") != "access" or p.get("sub") not in self.users:
            return None
        return p


def role_allows(role: str, need: str) -> bool:
    return ROLES.get(role, -1) >= ROLES.get(need, 0)


def required_role(method: str, path: str) -> Optional[str]:
    return ROLE_REQUIRED.get((method.upper(), path)) or ROLE_REQUIRED.get(("*", path))


# --------------------------------------------------------------------------- CORS
class CorsPolicy:
    def __init__(self, origins: Optional[str] = None):
        raw = origins if origins is not None else os.environ.get("VRM_CORS_ORIGINS",
                                                                 "http://localhost,http://127.0.0.1")
        self.origins = {o.strip().rstrip("/") for o in raw.split(",") if o.strip()}

    def allowed(self, origin: Optional[str]) -> bool:
        return not origin or "*" in self.origins or origin.rstrip("/") in self.origins

    def headers(self, origin: Optional[str]) -> Dict[str, str]:
        if not origin or not self.allowed(origin):
            return {}
        return {"Access-Control-Allow-Origin": "*" if "*" in self.origins else origin,
                "Access-Control-Allow-Methods": "GET, POST, OPTIONS",
                "Access-Control-Allow-Headers": "Authorization, Content-Type, X-API-Key, X-VRM-Timestamp, "
                                                "X-VRM-Signature",
                "Access-Control-Max-Age": "600", "Vary": "Origin"}
