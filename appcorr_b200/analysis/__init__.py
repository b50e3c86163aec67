"""Offline analysis tools for serving logs: timelines, early-exit simulation, nsys re-timing."""
