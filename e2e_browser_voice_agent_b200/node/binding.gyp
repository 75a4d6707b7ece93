# node-gyp recipe of the N-API addon (UNVERIFIED: no Node.js in this build image).
#   cd e2e_browser_voice_agent_b200/node && npm install node-addon-api && npx node-gyp rebuild
# It links libh2cuda.so from the package directory (build it first with e2e_browser_voice_agent_b200/build.py).
{
  "targets": [{
    "target_name": "h2cuda",
    "sources": ["h2cuda_node.cc"],
    "include_dirs": ["<!@(node -p \"require('node-addon-api').include\")", "../../include"],
    "defines": ["NAPI_CPP_EXCEPTIONS"],
    "cflags_cc": ["-std=c++17", "-fexceptions"],
    "libraries": ["-L<(module_root_dir)/..", "-lh2cuda", "-Wl,-rpath,<(module_root_dir)/.."]
  }]
}
