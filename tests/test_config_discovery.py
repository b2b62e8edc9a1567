"""Configuration (defaults -> YAML -> VRM_* environment, live flag view, validation,
reload hooks) and node discovery (UDP announcements on localhost, static VRM_NODES,
expiry of silent nodes)."""
import socket
import time

from vramancer_b200.cluster import discovery
from vramancer_b200.utils import config


def test_flags_live_view(monkeypatch):
    monkeypatch.delenv("VRM_MAX_BATCH_SIZE", raising=False)
    assert config.flags.VRM_MAX_BATCH_SIZE == 64
    monkeypatch.setenv("VRM_MAX_BATCH_SIZE", "12")
    assert config.flags.VRM_MAX_BATCH_SIZE == 12
    monkeypatch.setenv("VRM_MAX_BATCH_SIZE", "not-a-number")
    assert config.flags.VRM_MAX_BATCH_SIZE == 64          # bad values fall back to the default
    monkeypatch.setenv("VRM_CUDA_GRAPH", "off")
    assert config.flags.VRM_CUDA_GRAPH is False
    names = {d["name"] for d in config.flags.describe()}
    assert {"VRM_API_TOKEN", "VRM_KV_CACHE_DTYPE", "VRM_PROMPT_LOOKUP"} <= names


def test_yaml_then_env_then_validation_and_reload(tmp_path, monkeypatch):
    p = tmp_path / "config.yaml"
    p.write_text("max_batch: 7\nport: 6000\nkv_cache_dtype: fp8\ncustom_key: 3\n")
    monkeypatch.setenv("VRM_CONFIG", str(p))
    monkeypatch.setenv("VRM_N_CTX", "2048")
    monkeypatch.delenv("VRM_MAX_BATCH_SIZE", raising=False)
    seen = []
    config.on_reload(seen.append)
    c = config.reload_config()
    assert (c.max_batch, c.port, c.kv_cache_dtype, c.max_model_len) == (7, 6000, "fp8", 2048)
    assert c.extra == {"custom_key": 3} and seen and seen[-1] is c
    monkeypatch.setenv("VRM_MAX_BATCH_SIZE", "3")        # the environment wins over the file
    assert config.reload_config().max_batch == 3
    assert config.get_config().validate() == []
    bad = config.Config(port=0, gpu_memory_utilization=2.0, max_batch=0, kv_cache_dtype="int4")
    assert len(bad.validate()) == 4
    monkeypatch.delenv("VRM_CONFIG")
    config.reload_config()


def _free_udp_port():
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_discovery_over_udp_and_static_nodes(monkeypatch):
    port = _free_udp_port()
    d = discovery.ClusterDiscovery(port=port, bind="127.0.0.1")
    assert d.start()
    try:
        assert discovery.announce("10.0.0.7", 5030, {"gpus": 8}, discovery_port=port, broadcast_addr="127.0.0.1")
        t0 = time.time()
        while time.time() - t0 < 5:
            urls = {n["url"]: n for n in discovery.known_nodes()}
            if "http://10.0.0.7:5030" in urls:
                break
            time.sleep(0.05)
        assert urls["http://10.0.0.7:5030"]["gpus"] == 8
    finally:
        d.stop()
    monkeypatch.setenv("VRM_NODES", "http://static-a:5030, http://static-b:5030")
    discovery.register_node("http://old:5030")
    discovery._nodes["http://old:5030"]["last_seen"] -= 100
    urls = {n["url"] for n in discovery.known_nodes(ttl_s=30)}
    assert {"http://static-a:5030", "http://static-b:5030"} <= urls and "http://old:5030" not in urls


def test_mdns_wire_format_roundtrip():
    from vramancer_b200.cluster import mdns
    r = mdns.MDNSResponder("node7", "10.0.0.7", 5030, {"model": "qwen2.5-14b", "gpus": 8})
    msg = mdns.parse_message(r.records())
    assert msg["response"]
    types = {rt: val for _, rt, _, _, val in msg["records"]}
    assert types[mdns.T_PTR] == "node7._vramancer._tcp.local."
    assert types[mdns.T_SRV][2] == 5030 and types[mdns.T_A] == "10.0.0.7"
    assert types[mdns.T_TXT]["model"] == "qwen2.5-14b" and types[mdns.T_TXT]["url"] == "http://10.0.0.7:5030"
    q = mdns.parse_message(mdns.build_query())
    assert q["questions"][0][:2] == (mdns.SERVICE_TYPE, mdns.T_PTR) and not q["response"]


def test_mdns_browse_finds_a_responder_on_loopback():
    from vramancer_b200.cluster import mdns
    port = _free_udp_port()
    r = mdns.MDNSResponder("b200-a", "10.1.2.3", 5031, {"gpus": 8}, group="127.0.0.1", mdns_port=port,
                           bind="127.0.0.1")
    assert r.start()
    try:
        found = mdns.browse(timeout=1.0, group="127.0.0.1", mdns_port=port)
        assert [f["url"] for f in found] == ["http://10.1.2.3:5031"]
        assert found[0]["gpus"] == "8" and found[0]["discovery"] == "mdns"
        assert any(n["url"] == "http://10.1.2.3:5031" for n in discovery.known_nodes())
        assert r.answered >= 1
    finally:
        r.stop()


def _free_udp_port():
    import socket
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_every_environment_variable_read_is_registered():
    """Each VRM_* variable the package reads (os.environ in Python, getenv in the CUDA /
    C++ sources) has a typed, documented registry entry; the reference's names for the
    same settings resolve through the aliases."""
    import pathlib
    import re

    from vramancer_b200.utils.config import FLAG_ALIASES, FLAG_REGISTRY, flags
    root = pathlib.Path(__file__).resolve().parents[1] / "vramancer_b200"
    pat = re.compile(r'(?:environ\.get|environ\[|getenv|_env)\(\s*"(VRM_[A-Z0-9_]+)"|environ\["(VRM_[A-Z0-9_]+)"\]')
    read = set()
    for f in list(root.rglob("*.py")) + list(root.rglob("*.cu")) + list(root.rglob("*.cpp")):
        for m in pat.finditer(f.read_text(errors="ignore")):
            read.add(m.group(1) or m.group(2))
    assert read, "no environment reads found"
    missing = sorted(read - set(FLAG_REGISTRY) - set(FLAG_ALIASES.values()))
    assert not missing, missing
    for name, (typ, default, cat, doc) in FLAG_REGISTRY.items():
        assert doc and cat and isinstance(default, typ) or default is None, name


def test_reference_flag_names_are_aliases(monkeypatch):
    from vramancer_b200.utils.config import flags
    monkeypatch.delenv("VRM_MAX_BODY_BYTES", raising=False)
    monkeypatch.setenv("VRM_MAX_BODY", "1234")
    assert flags.VRM_MAX_BODY_BYTES == 1234
    monkeypatch.setenv("VRM_MAX_BODY_BYTES", "99")
    assert flags.VRM_MAX_BODY_BYTES == 99
