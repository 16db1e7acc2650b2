"""Model Context Protocol client (stdio transport)."""
from .client import MCPStdioClient, MCPTool, MCPToolResult
