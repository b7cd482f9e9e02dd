"""HTTP front end (src/http.rs routes) without a GPU: the request checks that
answer before any device work, with the reference's status codes."""
import pytest

pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from fishai_engine.http import create_app, validate_model_path  # noqa: E402


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    d = tmp_path_factory.mktemp("models")
    return TestClient(create_app(model_dirs=[str(d)])), d


def test_health_and_status_without_model(client):
    c, _ = client
    h = c.get("/health").json()
    assert h["status"] == "ok" and h["model_loaded"] is False
    assert c.get("/api/model/status").json() == {"loaded": False, "config": None}


def test_sample_rejects_bad_requests(client):
    c, _ = client
    r = c.post("/api/sample", json={"logits": []})
    assert r.status_code == 400 and r.json()["code"] == 400
    r = c.post("/api/sample", json={"logits": [1.0, 2.0], "config": {"temperature": 2.5}})
    assert r.status_code == 400
    r = c.post("/api/sample", json={"logits": [1.0, 2.0], "config": {"top_p": 1.5}})
    assert r.status_code == 400
    r = c.post("/api/sample", json={"logits": [1.0, 2.0], "config": {"repetition_penalty": 0.0}})
    assert r.status_code == 400


def test_load_outside_allowed_dirs_is_forbidden(client, tmp_path):
    c, d = client
    outside = tmp_path / "x.gguf"
    outside.write_bytes(b"GGUF")
    r = c.post("/api/model/load", json={"path": str(outside)})
    assert r.status_code == 403 and r.json()["success"] is False
    assert validate_model_path(str(outside), []) == str(outside.resolve())
    inside = d / "y.gguf"
    inside.write_bytes(b"GGUF")
    assert validate_model_path(str(inside), [str(d)]) == str(inside.resolve())


def test_generate_without_model_is_unavailable(client):
    c, _ = client
    r = c.post("/api/model/generate", json={"prompt": "hi"})
    assert r.status_code == 503 and r.json()["success"] is False
    r = c.post("/api/model/generate/stream", json={"prompt": "hi"})
    assert r.status_code == 503


def test_unknown_route_is_404(client):
    c, _ = client
    r = c.get("/api/nothing")
    assert r.status_code == 404
