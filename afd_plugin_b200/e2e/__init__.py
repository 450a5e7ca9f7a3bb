"""End-to-end serving scenarios: launch, health-wait, request, compare, tear down."""

from afd_plugin_b200.e2e.scenarios import SCENARIOS, Scenario, server_command

__all__ = ["SCENARIOS", "Scenario", "server_command"]
