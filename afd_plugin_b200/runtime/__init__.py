"""Role runtimes: engine, model runners, FFN loop, graphs, DBO, workers."""
