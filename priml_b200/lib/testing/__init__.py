"""Test helpers that ship with the package: resource markers and per-user directory isolation."""
