"""Deployment artifacts: the Helm chart's values and templates reference the server's real
routes, options and resources (reference charts/air-rs)."""
import os

import yaml

from air_rs.config import EngineConfig

ROOT = os.path.join(os.path.dirname(__file__), "..", "deploy", "helm", "air-rs-b200")


def test_values_map_onto_engine_config():
    v = yaml.safe_load(open(os.path.join(ROOT, "values.yaml")))
    env = {f"AIR_{k.upper()}": str(x).lower() if isinstance(x, bool) else str(x) for k, x in v["engine"].items()}
    cfg = EngineConfig.from_env(env)                     # every key is a real engine option
    assert cfg.max_batch == v["engine"]["max_batch"] and cfg.pressure_control is True
    assert yaml.safe_load(open(os.path.join(ROOT, "Chart.yaml")))["name"] == "air-rs-b200"


def test_templates_use_real_routes_and_gpu_resources():
    t = {f: open(os.path.join(ROOT, "templates", f)).read() for f in os.listdir(os.path.join(ROOT, "templates"))}
    dep = t["deployment.yaml"]
    assert dep.count("path: /health") == 3 and "nvidia.com/gpu" in dep and "/dev/shm" in dep
    assert "prometheus.io/path: /metrics" in dep and '"serve"' in dep
    assert "air_active_requests" in t["hpa.yaml"] and "PodDisruptionBudget" in t["pdb.yaml"]


def test_server_reads_api_keys_from_env(monkeypatch):
    from air_rs.cli import build_parser
    args = build_parser().parse_args(["serve", "-m", "x.gguf"])
    assert args.api_key is None and args.port == 8080
