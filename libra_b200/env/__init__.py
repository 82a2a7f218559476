"""Environments for the workflows: rewards/graders, tools (code sandbox, search), prompts."""
