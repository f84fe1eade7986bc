"""Agent plane: data sources, the dispatcher (agent-loop manager), agent loops."""
