"""Measurement: CUDA-event timing, work models, named shape suites."""
