"""Minimal Model Context Protocol client over stdio (JSON-RPC 2.0, one JSON
object per line).

Counterpart of complexity/mcp/client.py:16-125 (tool listing and tool calls
against an MCP server subprocess).  Implements ``initialize``, the
``notifications/initialized`` notification, ``tools/list`` and ``tools/call``.
"""
from __future__ import annotations

import json
import subprocess
import threading
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence


@dataclass
class MCPTool:
    name: str
    description: str = ""
    input_schema: Dict[str, Any] = field(default_factory=dict)


@dataclass
class MCPToolResult:
    content: List[Dict[str, Any]]
    is_error: bool = False

    @property
    def text(self) -> str:
        return "\n".join(c.get("text", "") for c in self.content if c.get("type") == "text")


class MCPStdioClient:
    PROTOCOL_VERSION = "2024-11-05"

    def __init__(self, command: Sequence[str], env: Optional[Dict[str, str]] = None,
                 timeout: float = 30.0):
        self.proc = subprocess.Popen(list(command), stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                     stderr=subprocess.DEVNULL, text=True, env=env, bufsize=1)
        self.timeout = timeout
        self._id = 0
        self._lock = threading.Lock()

    def _send(self, obj: Dict[str, Any]) -> None:
        self.proc.stdin.write(json.dumps(obj) + "\n")
        self.proc.stdin.flush()

    def request(self, method: str, params: Optional[Dict[str, Any]] = None) -> Any:
        with self._lock:
            self._id += 1
            rid = self._id
            self._send({"jsonrpc": "2.0", "id": rid, "method": method, "params": params or {}})
            while True:
                line = self.proc.stdout.readline()
                if not line:
                    raise RuntimeError("MCP server closed the connection")
                msg = json.loads(line)
                if msg.get("id") != rid:
                    continue  # notifications or other responses
                if "error" in msg:
                    raise RuntimeError(f"MCP error: {msg['error']}")
                return msg.get("result")

    def initialize(self, client_name: str = "complexity_framework_b200") -> Dict[str, Any]:
        res = self.request("initialize", {"protocolVersion": self.PROTOCOL_VERSION,
                                          "capabilities": {},
                                          "clientInfo": {"name": client_name, "version": "0.1"}})
        self._send({"jsonrpc": "2.0", "method": "notifications/initialized"})
        return res

    def list_tools(self) -> List[MCPTool]:
        res = self.request("tools/list") or {}
        return [MCPTool(t["name"], t.get("description", ""), t.get("inputSchema", {}))
                for t in res.get("tools", [])]

    def call_tool(self, name: str, arguments: Optional[Dict[str, Any]] = None) -> MCPToolResult:
        res = self.request("tools/call", {"name": name, "arguments": arguments or {}}) or {}
        return MCPToolResult(res.get("content", []), bool(res.get("isError", False)))

    def close(self) -> None:
        if self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def __enter__(self):
        self.initialize()
        return self

    def __exit__(self, *exc):
        self.close()
