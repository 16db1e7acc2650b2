"""API facade and MCP stdio client on CPU."""
import json
import sys
import textwrap

from complexity_framework_b200 import api
from complexity_framework_b200.mcp import MCPStdioClient


def test_api_model_roundtrip(tmp_path):
    m = api.Model.from_preset("tiny", device="cpu", hidden_size=64, num_hidden_layers=1,
                              num_attention_heads=4, num_key_value_heads=2, intermediate_size=64,
                              shared_intermediate_size=128, num_experts=4, top_k=2,
                              routing_strategy="modulo_cyclic")
    out = m.train(["hello world " * 20, "the quick brown fox " * 20] * 20, steps=3, batch_size=2,
                  seq_len=32)
    assert out["steps"] == 3
    txt = m.generate("hi", max_new_tokens=4)
    assert isinstance(txt, str)
    assert isinstance(m.chat([{"role": "user", "content": "hey"}], max_new_tokens=2), str)
    m.save(tmp_path / "m")
    m2 = api.load(str(tmp_path / "m"), device="cpu")
    assert m2.num_parameters() == m.num_parameters()


SERVER = textwrap.dedent('''
    import json, sys
    for line in sys.stdin:
        msg = json.loads(line)
        if "id" not in msg:
            continue
        m = msg["method"]
        if m == "initialize":
            res = {"protocolVersion": "2024-11-05", "capabilities": {"tools": {}},
                   "serverInfo": {"name": "t"}}
        elif m == "tools/list":
            res = {"tools": [{"name": "add", "description": "a+b",
                              "inputSchema": {"type": "object"}}]}
        elif m == "tools/call":
            a = msg["params"]["arguments"]
            res = {"content": [{"type": "text", "text": str(a["a"] + a["b"])}]}
        sys.stdout.write(json.dumps({"jsonrpc": "2.0", "id": msg["id"], "result": res}) + "\\n")
        sys.stdout.flush()
''')


def test_mcp_client(tmp_path):
    srv = tmp_path / "srv.py"
    srv.write_text(SERVER)
    with MCPStdioClient([sys.executable, str(srv)]) as c:
        tools = c.list_tools()
        assert tools[0].name == "add"
        assert c.call_tool("add", {"a": 2, "b": 3}).text == "5"
