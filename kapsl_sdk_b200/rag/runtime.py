"""Host side: connector runtimes, the client, and installed extensions.

* :class:`SidecarRuntime` — the connector is a child process speaking JSON
  lines on stdin/stdout; every request has a deadline (a hung connector
  raises ``TimeoutError`` and is killed instead of blocking the host).
* :class:`WasmRuntime` — a connector compiled to a WASI preview1 command
  module, run by the in-repo interpreter (``_native.wasm_run``): one
  instantiation per request, the request line on stdin, the last non-empty
  stdout line as the response, with the environment and preopened
  directories the workspace grants (reference: wasmtime in
  crates/kapsl-rag/src/runtime/mod.rs:198-331).
* :class:`ExtensionRegistry` / :class:`ExtensionManager` — install connector
  directories (``manifest.json`` + entrypoint), keep per-workspace configs,
  launch sidecars with validated environment and paths
  (reference: crates/kapsl-rag/src/extension/mod.rs:39-391).
"""
from __future__ import annotations

import json
import os
import queue
import re
import shutil
import subprocess
import sys
import threading
import uuid
from typing import Optional

from .protocol import ConnectorManifest, decode_response, encode_request


class SidecarRuntime:
    def __init__(self, argv: list, env: Optional[dict] = None, cwd: Optional[str] = None, timeout_s: float = 30.0):
        self.timeout_s = timeout_s
        self.proc = subprocess.Popen(argv, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                     text=True, env=env, cwd=cwd, bufsize=1)
        self._lines: "queue.Queue" = queue.Queue()
        self._reader = threading.Thread(target=self._read, daemon=True)
        self._reader.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self._lines.put(line)
        self._lines.put(None)

    def send(self, line: str) -> str:
        if self.proc.poll() is not None:
            raise ConnectionError(f"connector exited with code {self.proc.returncode}")
        self.proc.stdin.write(line + "\n")
        self.proc.stdin.flush()
        try:
            out = self._lines.get(timeout=self.timeout_s)
        except queue.Empty:
            self.close()
            raise TimeoutError(f"connector did not answer within {self.timeout_s} s")
        if out is None:
            raise ConnectionError("connector closed its output")
        return out

    def close(self) -> None:
        if self.proc.poll() is None:
            try:
                self.proc.stdin.close()
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()
                self.proc.wait()


class WasmRuntime:
    def __init__(self, path: str, env: Optional[dict] = None, preopens: Optional[list] = None,
                 timeout_s: float = 30.0, fuel: int = 4_000_000_000):
        """``preopens``: (host dir, guest path, read only) triples."""
        from .._ext import native

        self._native = native()
        with open(path, "rb") as f:
            self.module = f.read()
        self.env = []
        for k, v in (env or {}).items():
            if not k or "\0" in k or "\0" in str(v):
                raise ValueError("env key must be non-empty and key/value cannot contain NUL")
            self.env.append((str(k), str(v)))
        self.preopens = []
        for host, guest, ro in preopens or []:
            if not os.path.isabs(host):
                raise ValueError("preopened host path must be absolute")
            if not guest or not guest.startswith("/") or "\0" in guest:
                raise ValueError("preopened guest path must be absolute")
            self.preopens.append((str(host), str(guest), bool(ro)))
        self.timeout_s = timeout_s
        self.fuel = fuel
        self.last_stderr = b""

    def send(self, line: str) -> str:
        code, out, err = self._native.wasm_run(self.module, (line + "\n").encode(), self.env, self.preopens,
                                               self.fuel, self.timeout_s)
        self.last_stderr = err
        lines = [l for l in out.decode("utf-8").splitlines() if l.strip()]
        if not lines:
            raise ConnectionError(f"connector exited (code {code}) without a response: "
                                  f"{err.decode('utf-8', 'replace')[-300:]}")
        return lines[-1]

    def close(self) -> None:
        pass


class ConnectorClient:
    """Typed requests over a runtime; returns decoded results, raises
    ``ConnectorRemoteError`` when the connector answers Err."""

    def __init__(self, runtime):
        self.runtime = runtime

    def request(self, method: str, **params):
        rid = uuid.uuid4().hex
        _, _, value = decode_response(self.runtime.send(encode_request(rid, method, params)))
        return value

    def validate_config(self, config) -> None:
        self.request("ValidateConfig", config=config)

    def list_sources(self, config) -> list:
        return self.request("ListSources", config=config)

    def sync(self, source_id: str, cursor: Optional[str] = None) -> list:
        return self.request("Sync", source_id=source_id, cursor=cursor)

    def fetch_document(self, document_id: str):
        return self.request("FetchDocument", document_id=document_id)

    def transform_prompt(self, config, prompt: str) -> str:
        return self.request("TransformPrompt", config=config, prompt=prompt)

    def health(self) -> str:
        return self.request("Health")

    def shutdown(self) -> None:
        self.runtime.close()


# -------------------------------------------------------------- extensions
_ENV_KEY = re.compile(r"^[A-Za-z_][A-Za-z0-9_]*$")


def _validate_env(key: str, value: str) -> None:
    if not _ENV_KEY.match(key) or "\0" in value:
        raise ValueError(f"invalid environment entry {key!r}")


def _validate_rel_path(path: str) -> None:
    if os.path.isabs(path) or ".." in path.replace("\\", "/").split("/"):
        raise ValueError(f"path {path!r} must stay inside the extension directory")


class InstalledExtension:
    def __init__(self, path: str, manifest: ConnectorManifest):
        self.path, self.manifest = path, manifest

    @property
    def id(self) -> str:
        return self.manifest.id

    def entrypoint(self) -> str:
        ep = self.manifest.entrypoint or ("connector.py" if self.manifest.runtime == "sidecar" else "connector.wasm")
        _validate_rel_path(ep)
        full = os.path.join(self.path, ep)
        if not os.path.exists(full):
            raise FileNotFoundError(f"entrypoint {ep!r} missing in {self.path}")
        return full


def load_manifest(dir_path: str) -> ConnectorManifest:
    with open(os.path.join(dir_path, "manifest.json")) as f:
        return ConnectorManifest.from_json(json.load(f))


class ExtensionRegistry:
    def __init__(self, root: str):
        self.root = root

    def discover(self) -> list:
        out = []
        if not os.path.isdir(self.root):
            return out
        for name in sorted(os.listdir(self.root)):
            d = os.path.join(self.root, name)
            if os.path.isfile(os.path.join(d, "manifest.json")):
                out.append(InstalledExtension(d, load_manifest(d)))
        return out

    def install_from_dir(self, source: str) -> InstalledExtension:
        m = load_manifest(source)
        _validate_rel_path(m.id)
        dst = os.path.join(self.root, m.id)
        if os.path.exists(dst):
            shutil.rmtree(dst)
        shutil.copytree(source, dst)
        return InstalledExtension(dst, m)

    def uninstall(self, extension_id: str) -> None:
        _validate_rel_path(extension_id)
        d = os.path.join(self.root, extension_id)
        if not os.path.isdir(d):
            raise FileNotFoundError(f"extension {extension_id!r} is not installed")
        shutil.rmtree(d)


class ExtensionManager:
    """Per-workspace connector configs (``<config_root>/<workspace>/<connector>.json``)
    and sidecar launch."""

    def __init__(self, registry: ExtensionRegistry, config_root: str):
        self.registry, self.config_root = registry, config_root

    def _cfg_path(self, workspace: str, connector_id: str) -> str:
        _validate_rel_path(workspace)
        _validate_rel_path(connector_id)
        return os.path.join(self.config_root, workspace, f"{connector_id}.json")

    def set_workspace_config(self, workspace: str, connector_id: str, config: dict) -> None:
        p = self._cfg_path(workspace, connector_id)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        with open(p, "w") as f:
            json.dump(config, f)

    def get_workspace_config(self, workspace: str, connector_id: str) -> Optional[dict]:
        p = self._cfg_path(workspace, connector_id)
        if not os.path.exists(p):
            return None
        with open(p) as f:
            return json.load(f)

    def list_configs(self, workspace: str) -> list:
        d = os.path.join(self.config_root, workspace)
        return sorted(n[:-5] for n in os.listdir(d) if n.endswith(".json")) if os.path.isdir(d) else []

    def launch_connector(self, workspace: str, connector_id: str, timeout_s: float = 30.0) -> ConnectorClient:
        ext = {e.id: e for e in self.registry.discover()}.get(connector_id)
        if ext is None:
            raise FileNotFoundError(f"extension {connector_id!r} is not installed")
        cfg = self.get_workspace_config(workspace, connector_id) or {}
        if ext.manifest.runtime == "wasm":
            wasi = cfg.get("wasi") or {}
            preopens = [(d["host_path"], d["guest_path"], bool(d.get("read_only", False)))
                        for d in wasi.get("preopen_dirs") or []]
            return ConnectorClient(WasmRuntime(ext.entrypoint(), env=wasi.get("env") or {}, preopens=preopens,
                                               timeout_s=timeout_s))
        env = {"PATH": os.environ.get("PATH", "")}
        for k, v in (cfg.get("env") or {}).items():
            _validate_env(k, str(v))
            env[k] = str(v)
        ep = ext.entrypoint()
        argv = [sys.executable, ep] if ep.endswith(".py") else [ep]
        return ConnectorClient(SidecarRuntime(argv, env=env, cwd=ext.path, timeout_s=timeout_s))
