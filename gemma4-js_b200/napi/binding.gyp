{
  "targets": [
    {
      "target_name": "g4w4",
      "sources": ["g4w4_napi.c"],
      "include_dirs": ["../../include", "/usr/local/cuda/include"],
      "libraries": [
        "-L<(module_root_dir)/..", "-lg4w4", "-Wl,-rpath,<(module_root_dir)/..",
        "-L/usr/local/cuda/lib64", "-lcudart"
      ],
      "cflags": ["-std=c11", "-Wall", "-Wextra"]
    }
  ]
}
