"""Checkpoint loading and synthetic inputs."""
